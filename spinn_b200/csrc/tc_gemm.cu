// tc_gemm.cu -- implicit-GEMM convolution and plain GEMM on 5th-generation tensor cores.
//
//   Y[M][N] = epilogue( A[M][K] * W[N][K]^T )          (tf32 operands, fp32 accumulate)
//
// A is either the im2col view of an NHWC activation, fetched tap by tap with TMA in
// im2col mode (no im2col buffer exists anywhere), or a plain row-major matrix fetched with
// tiled TMA.  W is the weight matrix, K-major, zero-padded to a multiple of 32 columns.
// This replaces the reference's im2col copy + packed AVX2 GEMM
// (SPINN/run_time/ops/conv/conv2d.c:49-79,172-225, ops/mm/gemm_kernel.c:346-590) and its
// epilogue (gemm_kernel.c:316-338), which here runs on the accumulator before the store.
//
// Structure (one persistent CTA per SM, 256 threads):
//   warp 0      TMA producer: STAGES-deep ring of (A 128x32, W BNx32) tiles in shared memory
//   warp 1      MMA issuer: 4 x tcgen05.mma (128 x BN x 8) per stage into TMEM
//   warp 2      TMEM allocator (2 accumulators x BN columns)
//   warps 4..7  epilogue: tcgen05.ld -> bias / residual / activation / tf32 rounding ->
//               swizzled shared staging -> TMA store; each warp owns 32 accumulator lanes
// Tiles are 128 output pixels x BN output channels, scheduled n-fastest so that CTAs running
// together share the activation tile in L2.  Two TMEM accumulators let the epilogue of one
// tile overlap the main loop of the next.
//
// Every wait on an mbarrier is bounded (ptx.cuh mbar_wait); on expiry the CTA drains what it
// issued, frees TMEM and returns with the device error flag set.
#include <algorithm>
#include <atomic>

#include "internal.h"
#include "ptx.cuh"

namespace spinn {

namespace {

constexpr int kBM = 128;       // tile rows (output pixels) = TMEM lanes
constexpr int kBK = 32;        // K elements per pipeline stage (128 bytes of fp32/tf32)
constexpr int kThreads = 256;
constexpr uint64_t kTimeoutNs = 4000000000ull;  // 4 s per wait; a stage takes microseconds
constexpr uint64_t kDrainNs = 200000000ull;
constexpr int kSmemBudget = 232448 - 2048;      // 227 KiB opt-in minus barriers and alignment slack

enum AMode { kIm2col = 0, kTiled = 1 };

struct TcParams {
  int M, N;
  int num_kb;
  int cpad, taps, kw, dil_h, dil_w;
  int ohw, ow, stride_h, stride_w, pad_h, pad_w;
  int tiles_n, num_tiles;
  int has_res, act, round_out;
  float alpha;
  const float* bias;
  int* err;
};

template <int BN, int CB, bool RES>
struct Cfg {
  static constexpr int NSUB = kBK / CB;
  static constexpr uint32_t A_SUB = kBM * CB * 4;
  static constexpr uint32_t B_SUB = BN * CB * 4;
  static constexpr uint32_t A_STAGE = kBM * kBK * 4;
  static constexpr uint32_t B_STAGE = BN * kBK * 4;
  static constexpr uint32_t STAGE = A_STAGE + B_STAGE;
  // epilogue: two 32x32 fp32 staging blocks per epilogue warp (double-buffered TMA stores)
  static constexpr uint32_t OUT_BYTES = 2 * 4 * 4096;
  // residual ring: 128 rows x 32 columns per slot, filled by the residual producer warp
  static constexpr int RES_SLOTS = RES ? 3 : 0;
  static constexpr uint32_t RES_SLOT = kBM * 32 * 4;
  static constexpr uint32_t EPI = OUT_BYTES + RES_SLOTS * RES_SLOT;
  static constexpr int STAGES_FIT = (kSmemBudget - (int)EPI) / (int)STAGE;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // BN in {64,128,256} -> 128/256/512, powers of two
  static constexpr uint32_t SMEM = STAGES * STAGE + EPI + 256 + 1024;
  static_assert(STAGES >= 2, "pipeline needs two stages");
};

// Descriptor of the j-th 8-wide K slice of a stage whose rows are `rows` long in the MMA's
// M or N dimension.
template <int CB>
__device__ __forceinline__ uint64_t stage_desc(uint32_t stage_addr, int j, uint32_t sub_bytes) {
  if constexpr (CB == 4) {
    // no swizzle: core matrices of 8 rows x 16 B; the two 16-B K halves of one MMA live in
    // consecutive sub-tiles (LBO = sub-tile size), 8-row groups are 128 B apart (SBO).
    return make_smem_desc(stage_addr + (2 * j) * sub_bytes, sub_bytes, 128, kSwNone);
  } else {
    constexpr uint32_t row_bytes = CB * 4;
    const uint32_t sub = (8 * j) / CB;
    const uint32_t off = ((8 * j) % CB) * 4;
    constexpr uint32_t layout = CB == 32 ? kSw128 : CB == 16 ? kSw64 : kSw32;
    return make_smem_desc(stage_addr + sub * sub_bytes + off, 16, 8 * row_bytes, layout);
  }
}

template <int BN, int CB, int MODE, bool RES>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapY, const __grid_constant__ CUtensorMap mapR,
                   const TcParams p) {
  using C = Cfg<BN, CB, RES>;
  constexpr int STAGES = C::STAGES;
  constexpr int NRS = C::RES_SLOTS > 0 ? C::RES_SLOTS : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * C::A_STAGE;
  uint8_t* sOut = sB + STAGES * C::B_STAGE;  // [2][4 warps][4 KiB], 1024-aligned
  uint8_t* sRes = sOut + C::OUT_BYTES;       // [RES_SLOTS][16 KiB]
  uint64_t* full = reinterpret_cast<uint64_t*>(sRes + C::RES_SLOTS * C::RES_SLOT);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rfull = tempty + 2;
  uint64_t* rempty = rfull + NRS;
  uint64_t* drain = rempty + NRS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    for (int r = 0; r < NRS; ++r) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&mapA);
    prefetch_tmap(&mapB);
    prefetch_tmap(&mapY);
    if constexpr (RES) prefetch_tmap(&mapR);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (A, W)
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t armed = 0, armed_ph = 0;  // bit s: stage s armed at least once; its last parity
      for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
        const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
        const int m0 = tm * kBM, n0 = tn * BN;
        int w0 = 0, h0 = 0, img = 0;
        if constexpr (MODE == kIm2col) {
          img = m0 / p.ohw;
          const int rem = m0 - img * p.ohw;
          const int oh = rem / p.ow, ow = rem - oh * p.ow;
          w0 = ow * p.stride_w - p.pad_w;
          h0 = oh * p.stride_h - p.pad_h;
        }
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, kTimeoutNs)) break;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          armed |= 1u << s;
          armed_ph = (armed_ph & ~(1u << s)) | (ph << s);
          uint8_t* a_dst = sA + s * C::A_STAGE;
          uint8_t* b_dst = sB + s * C::B_STAGE;
#pragma unroll
          for (int j = 0; j < C::NSUB; ++j) {
            const int k = kb * kBK + j * CB;
            if constexpr (MODE == kIm2col) {
              int tap = k / p.cpad;
              const int c0 = k - tap * p.cpad;
              if (tap >= p.taps) tap = p.taps - 1;  // K padding: any real tap, its weights are zero
              const int r = tap / p.kw, q = tap - r * p.kw;
              tma_load_im2col_4d(&mapA, &full[s], a_dst + j * C::A_SUB, c0, w0, h0, img,
                                 (uint16_t)(q * p.dil_w), (uint16_t)(r * p.dil_h));
            } else {
              tma_load_2d(&mapA, &full[s], a_dst + j * C::A_SUB, k, m0);
            }
            tma_load_2d(&mapB, &full[s], b_dst + j * C::B_SUB, k, n0);
          }
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (*abort_flag) {
        // Let every copy this thread issued land before the CTA's shared memory goes away.
        volatile int dummy = 0;
        for (int st = 0; st < STAGES; ++st)
          if (armed & (1u << st)) mbar_wait(&full[st], (armed_ph >> st) & 1, &dummy, kDrainNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_tf32(kBM, BN);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool issued = false;
      for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++it) {
        const int b = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[b], aph ^ 1, abort_flag, kTimeoutNs)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + b * BN;
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, kTimeoutNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * C::A_STAGE);
          const uint32_t b0 = smem_u32(sB + s * C::B_STAGE);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            umma_tf32(d, stage_desc<CB>(a0, j, C::A_SUB), stage_desc<CB>(b0, j, C::B_SUB), idesc,
                      (kb | j) != 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      if (*abort_flag && issued) {
        volatile int dummy = 0;
        umma_commit(drain);
        mbar_wait(drain, 0, &dummy, kDrainNs);
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ residual producer
    // Streams the residual, 128 rows x 32 columns per slot, ahead of the epilogue so the
    // loads overlap the main loop instead of sitting on the epilogue's critical path.
    if constexpr (RES) {
      if (lane == 0) {
        int slot = 0;
        uint32_t ph = 0;
        uint32_t armed = 0, armed_ph = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
          const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
          const int m0 = tm * kBM, n0 = tn * BN;
          bool ok = true;
          for (int c = 0; c < BN / 32 && n0 + c * 32 < p.N; ++c) {
            if (!mbar_wait(&rempty[slot], ph ^ 1, abort_flag, kTimeoutNs)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&rfull[slot], C::RES_SLOT);
            armed |= 1u << slot;
            armed_ph = (armed_ph & ~(1u << slot)) | (ph << slot);
            tma_load_2d(&mapR, &rfull[slot], sRes + slot * C::RES_SLOT, n0 + c * 32, m0);
            if (++slot == C::RES_SLOTS) {
              slot = 0;
              ph ^= 1;
            }
          }
          if (!ok) break;
        }
        if (*abort_flag) {
          volatile int dummy = 0;
          for (int r = 0; r < C::RES_SLOTS; ++r)
            if (armed & (1u << r)) mbar_wait(&rfull[r], (armed_ph >> r) & 1, &dummy, kDrainNs);
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;  // TMEM lane quarter this warp may access
    int rslot = 0;
    uint32_t rph = 0;
    uint32_t chunk_no = 0;  // selects the output staging buffer
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
      const int m0 = tm * kBM, n0 = tn * BN;
      const int b = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      mbar_wait(&tfull[b], aph, abort_flag, kTimeoutNs);
      __syncwarp();
      if (*abort_flag) break;
      tc_fence_after();
      const int row0 = m0 + wq * 32;
      const bool rows_live = row0 < p.M;
      for (int c = 0; c < BN / 32; ++c) {
        const int col0 = n0 + c * 32;
        if (col0 >= p.N) break;
        const float* res_row = nullptr;
        if constexpr (RES) {
          mbar_wait(&rfull[rslot], rph, abort_flag, kTimeoutNs);
          __syncwarp();
          if (*abort_flag) break;
          res_row = reinterpret_cast<const float*>(sRes + rslot * C::RES_SLOT) + (wq * 32 + lane) * 32;
        }
        if (rows_live) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + b * BN + c * 32 + ((uint32_t)(wq * 32) << 16), r);
          tmem_ld_wait();
          const float bias_lane = (p.bias && col0 + lane < p.N) ? __ldg(p.bias + col0 + lane) : 0.0f;
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = p.alpha * __uint_as_float(r[i]) + __shfl_sync(0xffffffffu, bias_lane, i);
          if constexpr (RES) {
            const int rr = wq * 32 + lane;  // row inside the 128-row residual slot
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 x = *reinterpret_cast<const float4*>(res_row + ((j ^ (rr & 7)) * 4));
              v[4 * j + 0] += x.x;
              v[4 * j + 1] += x.y;
              v[4 * j + 2] += x.z;
              v[4 * j + 3] += x.w;
            }
          }
          if (p.act == 1 || p.act == 5) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = v[i] < 0.0f ? 0.0f : v[i];
          } else if (p.act == 3) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = v[i] / (1.0f + expf(-v[i]));
          }
          if (p.round_out) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = to_tf32_rna(v[i]);
          }
          float* st_out = reinterpret_cast<float*>(sOut + ((chunk_no & 1) * 4 + wq) * 4096);
          if (lane == 0) tma_store_wait_read<1>();  // the store that used this buffer has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            *reinterpret_cast<float4*>(st_out + lane * 32 + ((j ^ (lane & 7)) * 4)) =
                make_float4(v[4 * j + 0], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&mapY, st_out, col0, row0);
            tma_store_commit();
          }
          ++chunk_no;
        }
        if constexpr (RES) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&rempty[rslot]);
          if (++rslot == C::RES_SLOTS) {
            rslot = 0;
            rph ^= 1;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if (lane == 0) tma_store_wait0();
    __syncwarp();
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && p.err) atomicExch(p.err, 1);
}

template <int BN, int CB, int MODE, bool RES>
int launch_variant(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my, const CUtensorMap& mr,
                   const TcParams& p, int grid, cudaStream_t stream) {
  using C = Cfg<BN, CB, RES>;
  auto kern = tc_gemm_kernel<BN, CB, MODE, RES>;
  // The opt-in shared-memory size is a per-device function attribute: set it once per device.
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  SPINN_CUDA_TRY(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    SPINN_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    configured.fetch_or(bit);
  }
  kern<<<grid, kThreads, C::SMEM, stream>>>(ma, mb, my, mr, p);
  SPINN_CUDA_TRY(cudaGetLastError());
  return 0;
}

template <int MODE, bool RES>
int dispatch_bn_cb(int bn, int cb, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my,
                   const CUtensorMap& mr, const TcParams& p, int grid, cudaStream_t s) {
#define SPINN_TC_CASE(BNV, CBV) \
  if (bn == BNV && cb == CBV) return launch_variant<BNV, CBV, MODE, RES>(ma, mb, my, mr, p, grid, s);
  SPINN_TC_CASE(256, 32) SPINN_TC_CASE(128, 32) SPINN_TC_CASE(64, 32)
  if constexpr (MODE == kIm2col) {
    SPINN_TC_CASE(256, 16) SPINN_TC_CASE(128, 16) SPINN_TC_CASE(64, 16)
    SPINN_TC_CASE(256, 8) SPINN_TC_CASE(128, 8) SPINN_TC_CASE(64, 8)
    SPINN_TC_CASE(256, 4) SPINN_TC_CASE(128, 4) SPINN_TC_CASE(64, 4)
  }
#undef SPINN_TC_CASE
  set_error("tcgen05 gemm: no variant for BN=%d CB=%d mode=%d", bn, cb, MODE);
  return SPINN_CUDA_EUNSUPPORTED;
}

// Bounding box of the im2col traversal.  Base pixel of output (oy, ox) is
// (oy*sh - ph, ox*sw - pw); the traversal walks base positions lower..(extent-1+upper) in
// steps of the stride, so upper is chosen to make it visit exactly oh x ow positions
// (independent of bottom/right padding and of floor division in the output size).
void im2col_corners(const TcGemmArgs& a, int* lw, int* lh, int* uw, int* uh) {
  *lw = -a.pw;
  *lh = -a.ph;
  *uw = (a.ow - 1) * a.sw - a.pw - a.w + 1;
  *uh = (a.oh - 1) * a.sh - a.ph - a.h + 1;
}

int channel_block(int cpad) {
  for (int cb : {32, 16, 8, 4})
    if (cpad % cb == 0) return cb;
  return 0;
}

CUtensorMapSwizzle swizzle_for(int cb) {
  return cb == 32 ? CU_TENSOR_MAP_SWIZZLE_128B
                  : cb == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : cb == 8 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
}

int choose_bn(int M, int N, int sms) {
  // Cost model: waves of tiles times the per-tile time; narrow tiles pay a shared-memory
  // bandwidth penalty (the W tile is re-read per 8-wide K step for fewer output columns).
  const int cands[3] = {256, 128, 64};
  int best = 256;
  double best_cost = 1e300;
  const int tm = (M + kBM - 1) / kBM;
  for (int bn : cands) {
    if (bn > 64 && bn >= 2 * ((N + 63) / 64) * 64) continue;  // far wider than N
    const int tn = (N + bn - 1) / bn;
    const long tiles = (long)tm * tn;
    const long waves = (tiles + sms - 1) / sms;
    const double per_tile = bn == 256 ? 256.0 : bn == 128 ? 128.0 * 1.15 : 64.0 * 1.6;
    const double cost = waves * per_tile;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace

bool tc_gemm_supported(const TcGemmArgs& a, std::string* why) {
  auto fail = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (a.N <= 0 || a.M <= 0) return fail("empty problem");
  if (a.ldy % 4 != 0 || a.ldy < a.N) return fail("output row stride must be a multiple of 4 floats");
  if ((reinterpret_cast<uintptr_t>(a.y) & 15) || (reinterpret_cast<uintptr_t>(a.wt) & 15) ||
      (reinterpret_cast<uintptr_t>(a.x) & 15))
    return fail("operand not 16-byte aligned");
  if (a.res && (a.ldr % 4 != 0 || (reinterpret_cast<uintptr_t>(a.res) & 15))) return fail("residual misaligned");
  if (a.kpad % 32 != 0) return fail("weight K padding must be a multiple of 32");
  if (a.a_mode == 0) {
    if (channel_block(a.cpad) == 0) return fail("channel count must be a multiple of 4");
    if (a.sh > 8 || a.sw > 8 || a.sh < 1 || a.sw < 1) return fail("stride out of TMA range");
    int lw, lh, uw, uh;
    im2col_corners(a, &lw, &lh, &uw, &uh);
    if (a.oh < 1 || a.ow < 1 || a.M != a.n * a.oh * a.ow) return fail("output geometry inconsistent");
    if (lw < -128 || lh < -128 || uw < -128 || uh < -128 || lw > 127 || lh > 127 || uw > 127 || uh > 127)
      return fail("padding outside the im2col corner range");
    if ((a.kw - 1) * a.dw > 65535 || (a.kh - 1) * a.dh > 65535) return fail("filter offset too large");
    if ((long)a.kh * a.kw * a.cpad > a.kpad) return fail("weight K smaller than the filter volume");
  } else {
    if (a.lda % 4 != 0 || a.lda < a.K) return fail("A row stride must be a multiple of 4 floats");
    if (a.kpad < a.K) return fail("weight K smaller than K");
  }
  return true;
}

int tc_gemm_launch(const TcGemmArgs& a, cudaStream_t stream) {
  std::string why;
  if (!tc_gemm_supported(a, &why)) {
    set_error("tcgen05 gemm: %s", why.c_str());
    return SPINN_CUDA_EINVAL;
  }
  int dev = 0;
  SPINN_CUDA_TRY(cudaGetDevice(&dev));
  const int sms = sm_count(dev);
  TcParams p{};
  p.M = a.M;
  p.N = a.N;
  int cb = 32;
  CUtensorMap ma, mb, my, mr;
  int rc;
  if (a.a_mode == 0) {
    cb = channel_block(a.cpad);
    const int K = a.kh * a.kw * a.cpad;
    p.num_kb = tc_num_kb(K);
    p.cpad = a.cpad;
    p.taps = a.kh * a.kw;
    p.kw = a.kw;
    p.dil_h = a.dh;
    p.dil_w = a.dw;
    p.ohw = a.oh * a.ow;
    p.ow = a.ow;
    p.stride_h = a.sh;
    p.stride_w = a.sw;
    p.pad_h = a.ph;
    p.pad_w = a.pw;
    int lw, lh, uw, uh;
    im2col_corners(a, &lw, &lh, &uw, &uh);
    rc = encode_im2col_4d(&ma, a.x, a.n, a.h, a.w, a.cpad, lw, lh, uw, uh, cb, kBM, a.sw, a.sh, swizzle_for(cb));
    if (rc) return rc;
  } else {
    p.num_kb = tc_num_kb(a.K);
    p.cpad = a.K;
    p.taps = 1;
    p.kw = 1;
    rc = encode_tiled_2d(&ma, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.lda * 4, 32, kBM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (p.num_kb * 32 > a.kpad) {
    set_error("tcgen05 gemm: weights padded to %d, need %d", a.kpad, p.num_kb * 32);
    return SPINN_CUDA_EINVAL;
  }
  const int bn = a.bn ? a.bn : choose_bn(a.M, a.N, sms);
  rc = encode_tiled_2d(&mb, a.wt, (uint64_t)a.kpad, (uint64_t)a.N, (uint64_t)a.kpad * 4, (uint32_t)cb,
                       (uint32_t)bn, swizzle_for(cb));
  if (rc) return rc;
  rc = encode_tiled_2d(&my, a.y, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.ldy * 4, 32, 32,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (a.res) {
    rc = encode_tiled_2d(&mr, a.res, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.ldr * 4, 32, kBM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    mr = my;
  }
  p.tiles_n = (a.N + bn - 1) / bn;
  const long tiles = (long)((a.M + kBM - 1) / kBM) * p.tiles_n;
  if (tiles > 0x7FFFFFFF) {
    set_error("tcgen05 gemm: too many tiles");
    return SPINN_CUDA_EINVAL;
  }
  p.num_tiles = (int)tiles;
  p.has_res = a.res != nullptr;
  p.act = a.act;
  p.round_out = a.round_out;
  p.alpha = a.alpha;
  p.bias = a.bias;
  p.err = a.err ? a.err : device_error_flag(dev);
  const int grid = (int)std::min<long>(tiles, sms);
  if (a.a_mode == 0)
    return a.res ? dispatch_bn_cb<kIm2col, true>(bn, cb, ma, mb, my, mr, p, grid, stream)
                 : dispatch_bn_cb<kIm2col, false>(bn, cb, ma, mb, my, mr, p, grid, stream);
  return a.res ? dispatch_bn_cb<kTiled, true>(bn, cb, ma, mb, my, mr, p, grid, stream)
               : dispatch_bn_cb<kTiled, false>(bn, cb, ma, mb, my, mr, p, grid, stream);
}

}  // namespace spinn
