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
// Structure (one persistent CTA per SM, 384 threads):
//   warp 0      TMA producer: STAGES-deep ring of (A 128xBK, W BNxBK) tiles in shared memory
//               (resident-weight variants: W loaded once, the ring carries A only)
//   warp 1      MMA issuer: BK/8 x tcgen05.mma (128 x BN x 8) per stage and M sub-tile into TMEM
//   warp 2      TMEM allocator (all 512 columns)
//   warp 3      residual producer (fused residual variants)
//   warps 4..11 epilogue: tcgen05.ld -> bias / residual / activation / tf32 rounding ->
//               swizzled shared staging -> TMA store; warps w and w+4 share the 32
//               accumulator lanes of quarter w % 4 and take alternate 32-column chunks
//               (with two M sub-tiles: warps 4..7 drain sub-tile 0, warps 8..11 sub-tile 1)
// Tiles are 128 output pixels x BN output channels (256 pixels for CTA pairs and for two M
// sub-tiles), scheduled n-fastest so that CTAs running together share the activation tile in
// L2.  The TMEM accumulators (all 512 columns: 512 / (BN x sub-tiles) of them) let the
// epilogue of one tile overlap the main loop of the next ones.
//
// Problems with fewer tiles than SMs (small batches, the last stages of a ResNet, the FC
// layer) are split along K when the caller supplies a workspace: each (tile, K slice) unit
// stores raw fp32 partials into its own plane of the workspace and splitk_finish_kernel sums
// the planes in a fixed order and applies the epilogue, so results are deterministic.
//
// Every wait on an mbarrier is bounded (ptx.cuh mbar_wait); on expiry the CTA drains what it
// issued, frees TMEM and returns with the device error flag set.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace spinn {

namespace {

constexpr int kBM = 128;       // tile rows (output pixels) = TMEM lanes
constexpr uint64_t kTimeoutNs = 4000000000ull;  // 4 s per wait; a stage takes microseconds
constexpr uint64_t kDrainNs = 200000000ull;
constexpr int kSmemBudget = 232448 - 2048;      // 227 KiB opt-in minus barriers and alignment slack
constexpr int kWPrefetchKb = 1;                 // W k-blocks of the first unit warmed in L2 before the wait

enum AMode { kIm2col = 0, kTiled = 1 };

// The A operand's tensor maps: one per part when A is the channel concatenation of up to four
// NHWC tensors (a Concat that only this convolution reads is never materialised; each channel
// block of K is fetched from the part holding it).
constexpr int kMaxAParts = 4;
struct AMaps {
  CUtensorMap m[kMaxAParts];
};

struct TcParams {
  int M, N;
  int num_kb;
  int cpad, taps, kw, dil_h, dil_w;
  int ohw, ow, stride_h, stride_w, pad_h, pad_w;
  int tiles_n, num_tiles;
  int ksplit, kb_per, num_units;  // work unit u: tile u % num_tiles, z = u / num_tiles
  int batch, b_batched;           // batched GEMM: z is the batch index (then ksplit == 1)
  int reverse;                    // walk the tiles from the last one (alternates between layers)
  int nstages;                    // ring stages in use (<= the variant's STAGES)
  int has_res, act, round_out;
  float alpha;
  const float* bias;
  int* err;
  int nparts;                // tensor maps of A in use (1 = an ordinary tensor)
  int part_c0[kMaxAParts];   // first channel (K column) of each part
  // Stream-K (sk = 1; batch 1, no split, no residual, no resident weights): worker w of
  // G = gridDim.x / PAIR owns k-blocks [w T / G, (w+1) T / G) of the T = num_tiles * num_kb
  // k-blocks laid out tile after tile.  A worker whose range starts inside a tile stores that
  // first piece raw into its slot of sk_ws and counts it done on sk_flags[w * PAIR + rank];
  // the worker holding the tile's first k-block adds those slots in worker order.
  int sk;
  float* sk_ws;
  int* sk_flags;
};

// One piece of a CTA's work: k-blocks [kb0, kb1) of a tile.  kind 0: the whole reduction of
// the tile (the ordinary epilogue); 1: a stream-K tail piece (raw partial to the worker's slot);
// 2: the head piece of a tile that later workers finish (adds their partials first).
struct Piece {
  int tile, z, kb0, kb1, kind;
};
// Arrivals on a stream-K flag: each epilogue warp of the producing CTA once, then each
// epilogue warp of the consuming CTA once; the last consumer arrival clears the flag.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Part of A holding channel (K column) c, and c relative to that part.
__device__ __forceinline__ int a_part(const TcParams& p, int* c) {
  int pi = 0;
#pragma unroll
  for (int q = 1; q < kMaxAParts; ++q)
    if (q < p.nparts && *c >= p.part_c0[q]) pi = q;
  *c -= p.part_c0[pi];
  return pi;
}

// BK: K depth of one pipeline stage, 32 or 64.  Deeper stages halve the barrier handoffs per
// K (each handoff costs a few hundred cycles of single-thread latency); CTA pairs use 64 (one
// handoff feeds 1024 MMA cycles per SM), 256-wide single-CTA tiles keep 32 so that four
// stages fit beside the W tile.
//
// MS: M sub-tiles per CTA.  MS = 2 gives one CTA a 256 x BN unit computed as two 128-row MMA
// streams that share each W stage; A arrives in 256-row boxes.  A TMA box costs the same few
// hundred cycles of issue whether it holds 128 or 256 rows (measured on B200), so for narrow
// tiles (BN 64 / 128), whose main loop is bounded by box issue rather than by the tensor
// pipe, this doubles the bytes per box and halves the W boxes per output.
//
// WR: resident weights.  When one N tile covers all of N and W is small (the stems: 64 output
// channels, K <= 256), the whole W matrix is loaded once per CTA into shared memory and the
// ring carries only A boxes: half the TMA boxes per stage for the box-bound narrow tiles.
constexpr uint32_t kWresBytes = 64 * 1024;
template <int BN, int CB, bool RES, int PAIR, int BK_, int MS_ = 1, bool WR_ = false>
struct Cfg {
  static constexpr int BK = BK_;
  static constexpr int MS = MS_;
  static constexpr bool WR = WR_;
  static constexpr uint32_t W_BYTES = WR ? kWresBytes : 0;
  static constexpr int AROWS = kBM * MS;  // A rows held by each CTA
  static constexpr int BNC = BN / PAIR;  // B rows (output channels) held by each CTA
  static constexpr int NSUB = BK / CB;   // TMA boxes per operand per stage
  static constexpr int KSTEPS = BK / 8;  // MMAs per stage (per M sub-tile)
  static constexpr uint32_t A_SUB = AROWS * CB * 4;
  static constexpr uint32_t B_SUB = BNC * CB * 4;
  static constexpr uint32_t A_STAGE = AROWS * BK * 4;
  static constexpr uint32_t B_STAGE = BNC * BK * 4;
  static constexpr uint32_t STAGE = A_STAGE + (WR ? 0 : B_STAGE);
  // Epilogue: groups of four warps (one per TMEM lane quarter); with two groups, group g
  // takes the 32-column chunks c with c % 2 == g.  The residual (128 rows x 32 columns per
  // slot, filled by the residual producer warp) goes through one ring per group -- a ring
  // shared by two groups would let one group wait on a slot two phases ahead of the other's,
  // which the parity test cannot tell apart.  256-wide residual tiles keep a single group
  // with a 3-slot ring: two 2-slot rings would leave too few stages beside a 256-wide W tile.
  // With MS = 2, group g drains M sub-tile g (all of its chunks).
  static constexpr int EPI_GROUPS = (RES && BN == 256) ? 1 : 2;
  static constexpr int EPI_WARPS = 4 * EPI_GROUPS;
  static constexpr int THREADS = 128 + 32 * EPI_WARPS;
  // output staging: 32x32 fp32 blocks, two per warp with one group, one per warp with two
  static constexpr int OUT_BUFS = 2 / EPI_GROUPS;
  static constexpr uint32_t OUT_BYTES = 8 * 4096;
  static constexpr int RES_G = !RES ? 0 : EPI_GROUPS == 1 ? 3 : 2;  // slots per group
  static constexpr int RES_SLOTS = RES_G * EPI_GROUPS;
  static constexpr uint32_t RES_SLOT = kBM * 32 * 4;
  static constexpr uint32_t EPI = OUT_BYTES + RES_SLOTS * RES_SLOT;
  static constexpr int STAGES_FIT = (kSmemBudget - (int)EPI - (int)W_BYTES) / (int)STAGE;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  // TMEM accumulators: all 512 columns, so narrow tiles (BN 128 / 64) get 4 / 8 buffers and
  // the MMA can run that many tiles ahead of the epilogue
  static constexpr int NACC = 512 / (BN * MS);
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t SMEM = STAGES * STAGE + W_BYTES + EPI + 512 + 1024;
  static_assert(STAGES >= 2, "pipeline needs two stages");
  static_assert(PAIR == 1 || BNC >= 64, "pair tiles split BN into halves of at least 64 rows");
  static_assert(MS == 1 || (PAIR == 1 && CB >= 16 && BN <= 128), "two M sub-tiles: narrow single-CTA tiles only");
  static_assert(!WR || (PAIR == 1 && !RES), "resident weights: single-CTA tiles without a fused residual");
  // Two TMA issuers for narrow single-CTA tiles when warp 3 is free (no residual ring, W in
  // the ring): warp 0 loads A and warp 3 loads W into the same stages.  One thread's TMA
  // issue stalls on the previous copies; two issuers raised a stream of 16 KiB boxes from
  // ~330 to ~240 cycles per box per SM.  (CTA pairs and 256-wide tiles measured slower.)
  static constexpr bool SPLIT_LOAD = !RES && !WR && PAIR == 1 && BN <= 128;
};

// Start-address offset (bytes) of the j-th 8-wide K slice of a stage, and the descriptor
// template (offset 0) for operand tiles with `sub_bytes` per channel block.
template <int CB>
__device__ __forceinline__ uint32_t kslice_offset(int j, uint32_t sub_bytes) {
  if constexpr (CB == 4) {
    return (2 * j) * sub_bytes;  // no swizzle: the two 16-B K halves of one MMA are consecutive sub-tiles
  } else {
    return ((8 * j) / CB) * sub_bytes + ((8 * j) % CB) * 4;
  }
}
template <int CB>
__device__ __forceinline__ uint64_t stage_desc0(uint32_t addr, uint32_t sub_bytes) {
  if constexpr (CB == 4) {
    // core matrices of 8 rows x 16 B; K halves sub_bytes apart (LBO), 8-row groups 128 B (SBO)
    return make_smem_desc(addr, sub_bytes, 128, kSwNone);
  } else {
    constexpr uint32_t layout = CB == 32 ? kSw128 : CB == 16 ? kSw64 : kSw32;
    return make_smem_desc(addr, 16, 8 * CB * 4, layout);
  }
}

// All lanes wait; the warp proceeds only if every lane saw the phase complete.  Warp-wide
// loops take every exit decision through these so that the lanes never diverge on a flag
// that another warp raises.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t ns) {
  const bool ok = mbar_wait(bar, parity, abort, ns);
  return __all_sync(0xffffffffu, ok);
}
__device__ __forceinline__ bool warp_aborted(volatile int* abort) { return __any_sync(0xffffffffu, *abort != 0); }
__device__ __forceinline__ bool warp_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t ns) {
  const bool ok = mbar_wait_backoff(bar, parity, abort, ns);
  return __all_sync(0xffffffffu, ok);
}
// Bounded warp-wide wait until the stream-K flag `f` reaches `target` arrivals (acquire: the
// partial sums published before those arrivals are visible afterwards).
__device__ __forceinline__ bool warp_wait_flag(const int* f, int target, volatile int* abort, uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (__all_sync(0xffffffffu, ld_acquire_gpu(f) >= target)) return true;
    if (warp_aborted(abort)) return false;
    if (__any_sync(0xffffffffu, globaltimer_ns() - t0 > ns)) {
      *abort = 1;
      return false;
    }
    __nanosleep(64);
  }
}

// A stream-K flag that nothing ever raises, and one warp that waits on it with the kernels'
// bounded wait: the wait must expire, raise the error word and return.
__device__ int g_flag_never_raised = 0;
__global__ void __launch_bounds__(32) flag_wait_expiry_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncwarp();
  if (!warp_wait_flag(&g_flag_never_raised, 1, &abort_flag, timeout_ns) && threadIdx.x == 0) atomicExch(err, 1);
}

// PAIR = 1: one CTA per 128 x BN tile.  PAIR = 2: a cluster of two CTAs per 256 x BN tile
// with one cta_group::2 MMA stream issued by the leader (rank 0); each CTA loads its own 128
// rows of A and BN/2 rows of W.  Barrier roles in pair mode: `full` of the leader counts the
// bytes of both CTAs; the leader's MMA thread signals `empty` and `tfull` in both CTAs; both
// CTAs' epilogue warps arrive on the leader's `tempty` (8 arrivals).
//
// The producer and MMA warps run their loops with all 32 lanes (lane 0 issues): a single
// diverged lane spends about half again as long per barrier handoff.
template <int BN, int CB, int MODE, bool RES, int PAIR, int BK_, int MS_, bool WR_>
__global__ void __launch_bounds__(Cfg<BN, CB, RES, PAIR, BK_, MS_, WR_>::THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ AMaps amaps, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapY, const __grid_constant__ CUtensorMap mapR,
                   const TcParams p) {
  using C = Cfg<BN, CB, RES, PAIR, BK_, MS_, WR_>;
  constexpr bool WR = C::WR;
  constexpr int STAGES = C::STAGES;
  constexpr int BK = C::BK;
  constexpr int MS = C::MS;
  constexpr int NRS = C::RES_SLOTS > 0 ? C::RES_SLOTS : 1;
  constexpr int TM = kBM * PAIR * MS;  // rows of one work unit
  // stream-K: 32-column chunks one epilogue warp drains per tile, and how many later workers'
  // partial sums (this CTA's rows) fit in the operand ring at once
  constexpr int SK_MYCH = MS == 2 ? BN / 32 : BN / 32 / C::EPI_GROUPS;
  constexpr int SK_NCAP = WR ? 0 : (int)((size_t)STAGES * C::STAGE / ((size_t)C::EPI_WARPS * SK_MYCH * 4096));
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * C::A_STAGE;
  uint8_t* sOut = sB + (WR ? C::W_BYTES : STAGES * C::B_STAGE);  // [OUT_BUFS][EPI_WARPS][4 KiB], 1024-aligned
  uint8_t* sRes = sOut + C::OUT_BYTES;       // [RES_SLOTS][16 KiB]
  uint64_t* full = reinterpret_cast<uint64_t*>(sRes + C::RES_SLOTS * C::RES_SLOT);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + C::NACC;
  uint64_t* rfull = tempty + C::NACC;
  uint64_t* rempty = rfull + NRS;
  uint64_t* drain = rempty + NRS;
  uint64_t* wfull = drain + 1;  // resident weights landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR == 2 ? cluster_ctarank() : 0;
  const int unit0 = blockIdx.x / PAIR, unit_step = gridDim.x / PAIR;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], C::SPLIT_LOAD ? 2 : 1);  // one expect_tx arrival per issuing warp
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::NACC; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], C::EPI_WARPS * PAIR);
    }
    for (int r = 0; r < NRS; ++r) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], 4);
    }
    mbar_init(drain, 1);
    mbar_init(wfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < p.nparts; ++i) prefetch_tmap(&amaps.m[i]);
    prefetch_tmap(&mapB);
    prefetch_tmap(&mapY);
    if constexpr (RES) prefetch_tmap(&mapR);
  }
  if (warp == 2) {
    if constexpr (PAIR == 2) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  // The weights do not depend on the previous kernel: warm L2 with the W boxes of this CTA's
  // first stage while that kernel finishes, so the first stage after the wait below hits L2.
  // (One stage only: prefetches occupy the SM's copy engine ahead of the loads that follow,
  // and eight stages' worth slowed the narrow YOLO-shaped layers by ~10%.  Resident weights
  // are loaded whole right after the wait anyway.)
  // Work of this CTA.  Ordinary launches: units unit0, unit0 + unit_step, ... (a dynamic
  // schedule -- units claimed from a global counter and handed to the other roles through a
  // shared-memory queue -- evened out the CTAs' finishing times but measured 1-2% slower end
  // to end).  Stream-K: consecutive tiles covering the worker's k-block range.
  const bool sk = !RES && !WR && p.sk != 0;
  const SkRange skr = sk ? sk_range(p.num_tiles, p.num_kb, unit0, unit_step) : SkRange{};
  auto get_piece = [&](int it, Piece& pc) -> bool {
    int t;
    if (sk) {
      if (!sk_piece(skr, it, &t, &pc.kb0, &pc.kb1, &pc.kind)) return false;
      pc.z = 0;
    } else {
      const long u = (long)unit0 + (long)it * unit_step;
      if (u >= p.num_units) return false;
      pc.z = (int)u / p.num_tiles;
      t = (int)u - pc.z * p.num_tiles;
      const int ks = p.batch > 1 ? 0 : pc.z;
      pc.kb0 = ks * p.kb_per;
      pc.kb1 = min(p.num_kb, pc.kb0 + p.kb_per);
      pc.kind = 0;
    }
    pc.tile = p.reverse ? p.num_tiles - 1 - t : t;
    return true;
  };
  Piece pc0;
  if (!WR && warp == (C::SPLIT_LOAD ? 3 : 0) && lane == 0 && get_piece(0, pc0)) {
    const int tn = pc0.tile % p.tiles_n;
    const int bzb = p.b_batched ? pc0.z : 0;
    const int kb0 = pc0.kb0, kb1 = min(pc0.kb1, kb0 + kWPrefetchKb);
    for (int kb = kb0; kb < kb1; ++kb)
#pragma unroll
      for (int j = 0; j < C::NSUB; ++j)
        tma_prefetch_3d(&mapB, kb * BK + j * CB, tn * BN + (int)rank * C::BNC, bzb);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) cluster_sync();  // the peer's barriers are initialised before use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above overlapped the previous kernel's tail; from here on its outputs (our
  // activations, residual) are visible and the buffers it read may be overwritten.
  griddep_wait();
  griddep_launch_dependents();

  auto take_unit = [&](int it) -> int {
    const long u = (long)unit0 + (long)it * unit_step;
    return u < p.num_units ? (int)u : -1;
  };

  if (warp == 0 || (C::SPLIT_LOAD && warp == 3)) {
    // ------------------------------------------------------------ TMA producer (A, W)
    // warp 0 issues A (and W unless split); with SPLIT_LOAD, warp 3 issues W; both walk the
    // same units and stages
    const bool do_a = warp == 0;
    const bool do_b = !WR && (C::SPLIT_LOAD ? warp == 3 : warp == 0);
    const uint32_t stage_tx = ((do_a ? C::A_STAGE : 0u) + (do_b ? C::B_STAGE : 0u)) * PAIR;
    int s = 0;
    uint32_t ph = 0;
    uint32_t armed = 0, armed_ph = 0;  // bit s: stage s armed at least once; its last parity
    // resident weights: all num_kb k-blocks of the single N tile, once, on `wfull`
    const bool w_issued = WR && do_a && get_piece(0, pc0);
    if (w_issued && lane == 0) {
      mbar_arrive_expect_tx(wfull, (uint32_t)p.num_kb * C::B_STAGE);
      for (int kb = 0; kb < p.num_kb; ++kb)
#pragma unroll
        for (int j = 0; j < C::NSUB; ++j)
          tma_load_3d(&mapB, wfull, sB + kb * C::B_STAGE + j * C::B_SUB, kb * BK + j * CB, 0, 0);
    }
    __syncwarp();
    for (int it = 0; !warp_aborted(abort_flag); ++it) {
      Piece pc;
      if (!get_piece(it, pc)) break;
      const int tile = pc.tile;
      const int bz = p.batch > 1 ? pc.z : 0;
      const int bzb = p.b_batched ? bz : 0;  // batch plane of W
      const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
      int m0 = tm * TM + (int)rank * kBM;
      if (m0 >= p.M) m0 = tm * TM;  // a pair's second half past the end: load valid rows, store none
      const int nb0 = tn * BN + (int)rank * C::BNC;
      const int kb0 = pc.kb0, kb1 = pc.kb1;
      int w0 = 0, h0 = 0, img = 0;
      // im2col walk state for the next box: channel offset c0 inside tap (r, q)
      int c0 = 0, r = 0, q = 0, tap = 0;
      if constexpr (MODE == kIm2col) {
        img = m0 / p.ohw;
        const int rem = m0 - img * p.ohw;
        const int oh = rem / p.ow, ow = rem - oh * p.ow;
        w0 = ow * p.stride_w - p.pad_w;
        h0 = oh * p.stride_h - p.pad_h;
        const int k0 = kb0 * BK;
        tap = k0 / p.cpad;
        c0 = k0 - tap * p.cpad;
        r = tap / p.kw;
        q = tap - r * p.kw;
      }
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!warp_wait(&empty[s], ph ^ 1, abort_flag, kTimeoutNs)) break;
        if (lane == 0) {
          if (rank == 0) mbar_arrive_expect_tx(&full[s], stage_tx);
          uint8_t* a_dst = sA + s * C::A_STAGE;
          uint8_t* b_dst = sB + s * C::B_STAGE;
          const uint32_t bar_leader = PAIR == 2 ? mapa_shared(smem_u32(&full[s]), 0) : 0;
#pragma unroll
          for (int j = 0; j < C::NSUB; ++j) {
            const int k = kb * BK + j * CB;
            if (!do_a) {
            } else if constexpr (MODE == kIm2col) {
              // K padding past the last tap: re-read the last tap, its weights are zero
              const int rr = tap < p.taps ? r : (p.taps - 1) / p.kw;
              const int qq = tap < p.taps ? q : (p.taps - 1) - ((p.taps - 1) / p.kw) * p.kw;
              int cc = tap < p.taps ? c0 : p.cpad - CB;
              const CUtensorMap* mapA = &amaps.m[a_part(p, &cc)];
              if constexpr (PAIR == 2)
                tma_load_im2col_4d_pair(mapA, bar_leader, a_dst + j * C::A_SUB, cc, w0, h0, img,
                                        (uint16_t)(qq * p.dil_w), (uint16_t)(rr * p.dil_h));
              else
                tma_load_im2col_4d(mapA, &full[s], a_dst + j * C::A_SUB, cc, w0, h0, img, (uint16_t)(qq * p.dil_w),
                                   (uint16_t)(rr * p.dil_h));
              c0 += CB;
              if (c0 == p.cpad) {
                c0 = 0;
                ++tap;
                if (++q == p.kw) {
                  q = 0;
                  ++r;
                }
              }
            } else {
              int kc = k;
              const CUtensorMap* mapA = &amaps.m[a_part(p, &kc)];
              if constexpr (PAIR == 2)
                tma_load_3d_pair(mapA, bar_leader, a_dst + j * C::A_SUB, kc, m0, bz);
              else
                tma_load_3d(mapA, &full[s], a_dst + j * C::A_SUB, kc, m0, bz);
            }
            if (do_b) {
              if constexpr (PAIR == 2)
                tma_load_3d_pair(&mapB, bar_leader, b_dst + j * C::B_SUB, k, nb0, bzb);
              else
                tma_load_3d(&mapB, &full[s], b_dst + j * C::B_SUB, k, nb0, bzb);
            }
          }
          if (rank == 0) {
            armed |= 1u << s;
            armed_ph = (armed_ph & ~(1u << s)) | (ph << s);
          }
        }
        __syncwarp();
        if (++s == p.nstages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    if (warp_aborted(abort_flag) && lane == 0) {
      // Let every copy this thread issued land before the CTA's shared memory goes away
      // (in a pair the leader's `full` also counts the peer's copies).
      volatile int dummy = 0;
      for (int st = 0; st < STAGES; ++st)
        if (armed & (1u << st)) mbar_wait(&full[st], (armed_ph >> st) & 1, &dummy, kDrainNs);
      if (w_issued) mbar_wait(wfull, 0, &dummy, kDrainNs);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (pair leader)
    if (rank == 0) {
      constexpr uint32_t idesc = make_idesc_tf32(kBM * PAIR, BN);
      const uint64_t adesc0 = stage_desc0<CB>(smem_u32(sA), C::A_SUB);
      const uint64_t bdesc0 = stage_desc0<CB>(smem_u32(sB), C::B_SUB);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool issued = false;
      for (;; ++it) {
        Piece pc;
        if (!get_piece(it, pc) || warp_aborted(abort_flag)) break;
        const int b = it % C::NACC;
        const uint32_t aph = (it / C::NACC) & 1;
        const int kb0 = pc.kb0, kb1 = pc.kb1;
        if (!warp_wait(&tempty[b], aph ^ 1, abort_flag, kTimeoutNs)) break;
        if (WR && it == 0 && !warp_wait(wfull, 0, abort_flag, kTimeoutNs)) break;  // resident weights
        tc_fence_after();
        const uint32_t d = tmem_base + b * (BN * MS);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!warp_wait(&full[s], ph, abort_flag, kTimeoutNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            // resident weights are indexed by the k-block, the ring by the stage
            const uint64_t as = adesc0 + ((s * C::A_STAGE) >> 4),
                           bs = bdesc0 + (((WR ? (uint32_t)kb : (uint32_t)s) * C::B_STAGE) >> 4);
#pragma unroll
            for (int j = 0; j < C::KSTEPS; ++j) {
              const uint64_t ad = as + (kslice_offset<CB>(j, C::A_SUB) >> 4);
              const uint64_t bd = bs + (kslice_offset<CB>(j, C::B_SUB) >> 4);
              const uint32_t acc = (kb != kb0 || j != 0) ? 1u : 0u;
              if constexpr (PAIR == 2) {
                umma_tf32_pair(d, ad, bd, idesc, acc);
              } else {
#pragma unroll
                for (int ms = 0; ms < MS; ++ms)  // sub-tile ms: A rows 128 ms.., accumulator columns BN ms..
                  umma_tf32(d + ms * BN, ad + ((uint64_t)(ms * kBM * CB * 4) >> 4), bd, idesc, acc);
              }
            }
            if constexpr (PAIR == 2) {
              umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 0));
              umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
            } else {
              umma_commit(&empty[s]);
            }
          }
          __syncwarp();
          issued = true;
          if (++s == p.nstages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        if (lane == 0) {
          if constexpr (PAIR == 2) {
            umma_commit_pair(mapa_shared(smem_u32(&tfull[b]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&tfull[b]), 1));
          } else {
            umma_commit(&tfull[b]);
          }
        }
        __syncwarp();
      }
      if (warp_aborted(abort_flag) && issued && lane == 0) {
        volatile int dummy = 0;
        if constexpr (PAIR == 2)
          umma_commit_pair(mapa_shared(smem_u32(drain), 0));
        else
          umma_commit(drain);
        mbar_wait(drain, 0, &dummy, kDrainNs);
      }
      __syncwarp();
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ residual producer
    // Streams the residual, 128 rows x 32 columns per slot, ahead of the epilogue so the
    // loads overlap the main loop instead of sitting on the epilogue's critical path.
    if constexpr (RES) {
      if (lane == 0) {
        int count[2] = {0, 0};  // chunks loaded so far for each epilogue group
        uint32_t armed = 0, armed_ph = 0;
        int it = 0;  // units so far: chunk c goes to epilogue group (c + it) % EPI_GROUPS
        for (;; ++it) {  // ksplit == 1: a unit is a tile
          const int t = take_unit(it);
          if (t < 0 || *abort_flag) break;
          const int tile = p.reverse ? p.num_tiles - 1 - t : t;
          const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
          const int m0 = tm * TM + (int)rank * kBM, n0 = tn * BN;
          bool ok = true;
          // chunk c goes to group (c + it) % EPI_GROUPS; with two M sub-tiles every chunk
          // goes to both groups, each its own sub-tile's 128 rows
          for (int c = 0; ok && c < BN / 32 && n0 + c * 32 < p.N; ++c) {
            for (int h = 0; h < MS; ++h) {
              const int g = MS == 2 ? h : (c + it) % C::EPI_GROUPS;
              const int slot = g * C::RES_G + count[g] % C::RES_G;
              const uint32_t ph = (count[g] / C::RES_G) & 1;
              if (!mbar_wait(&rempty[slot], ph ^ 1, abort_flag, kTimeoutNs)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&rfull[slot], C::RES_SLOT);
              armed |= 1u << slot;
              armed_ph = (armed_ph & ~(1u << slot)) | (ph << slot);
              tma_load_2d(&mapR, &rfull[slot], sRes + slot * C::RES_SLOT, n0 + c * 32, m0 + h * kBM);
              ++count[g];
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
    const int wq = warp & 3;         // TMEM lane quarter this warp may access
    const int eg = (warp - 4) >> 2;  // epilogue group
    int rcount = 0;                  // residual chunks this group has consumed
    uint32_t nstore = 0;             // stores issued by this warp (selects the staging buffer)
    int it = 0;
    // A split launch (ksplit > 1) stores raw partial sums into plane `ks` of the workspace;
    // the finish kernel applies the epilogue after reducing the planes.
    const bool partial = p.ksplit > 1;
    const bool unit_alpha = p.alpha == 1.0f;
    for (;; ++it) {
      Piece pc;
      if (!get_piece(it, pc)) break;
      const int z = pc.z;  // K slice or batch -> output plane
      const int tile = pc.tile;
      const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
      // stream-K tail piece: raw partial sums to this worker's slot, no epilogue
      const bool raw = partial || pc.kind == 1;
      const int m0 = tm * TM + (int)rank * kBM, n0 = tn * BN;
      const int b = it % C::NACC;
      const uint32_t aph = (it / C::NACC) & 1;
      // Chunk c of this unit belongs to group (c + it) % EPI_GROUPS: rotating the ownership
      // spreads units with a single live chunk (N <= 32) over both groups.
      const int eo = (eg + C::EPI_GROUPS - it % C::EPI_GROUPS) % C::EPI_GROUPS;
      // This warp's bias values for the unit (lane l: column n0 + 32 c + l of each chunk c it
      // owns), fetched before the accumulator wait so the load latency is hidden behind it.
      // With two M sub-tiles a group owns every chunk of its sub-tile.
      constexpr int MYCH = MS == 2 ? BN / 32 : BN / 32 / C::EPI_GROUPS;
      float bias_reg[MYCH];
#pragma unroll
      for (int i = 0; i < MYCH; ++i) {
        const int col = n0 + 32 * (MS == 2 ? i : i * C::EPI_GROUPS + eo) + lane;
        bias_reg[i] = (!raw && p.bias && col < p.N) ? __ldg(p.bias + col) : 0.0f;
      }
      if (!warp_wait_backoff(&tfull[b], aph, abort_flag, kTimeoutNs)) break;
      tc_fence_after();
      const int row0 = m0 + (MS == 2 ? eg * kBM : 0) + wq * 32;
      const bool rows_live = row0 < p.M;
      // stream-K slot layout: [chunk of 32 columns][lane quarter][column][row in quarter], so
      // that a warp's 32 rows of one column are one 128-byte line and its part of a chunk is
      // one contiguous 4 KiB block
      constexpr size_t kSlot = (size_t)kBM * MS * BN;
      const size_t sk_wbase = (size_t)(((MS == 2 ? eg * (BN / 32) : 0) * 4 + wq) * 1024);
      // Head of a split tile: the workers after this one whose ranges start inside the tile
      // (unit0 + 1 .. sk_j1 - 1) each left the rest of the tile's sum in their slots.  The
      // first SK_NCAP of them are copied into this warp's share of the operand ring -- idle
      // now, this is the CTA's last piece -- in one round trip, instead of one per chunk.
      int sk_j1 = unit0 + 1, sk_jfast = unit0 + 1;
      if (sk && pc.kind == 2) {
        bool ok = true;
        for (; ok && sk_contributes(skr, sk_j1, skr.t0 + it); ++sk_j1)
          ok = warp_wait_flag(p.sk_flags + sk_j1 * PAIR + rank, C::EPI_WARPS, abort_flag, kTimeoutNs);
        if (!ok) break;
        sk_jfast = min(sk_j1, unit0 + 1 + SK_NCAP);
        if (rows_live && sk_jfast > unit0 + 1) {
          float* stage = reinterpret_cast<float*>(sA) + (size_t)(warp - 4) * SK_NCAP * SK_MYCH * 1024;
          for (int j = unit0 + 1; j < sk_jfast; ++j) {
            const float* slot = p.sk_ws + (size_t)(j * PAIR + (int)rank) * kSlot + sk_wbase;
            for (int c = 0; c < BN / 32 && n0 + c * 32 < p.N; ++c) {
              if (MS == 1 && c % C::EPI_GROUPS != eo) continue;
              const float* src = slot + (size_t)c * 4096;
              float* dst = stage + ((j - unit0 - 1) * SK_MYCH + (MS == 2 ? c : c / C::EPI_GROUPS)) * 1024;
#pragma unroll
              for (int k = 0; k < 8; ++k) cp_async_16(dst + (k * 32 + lane) * 4, src + (k * 32 + lane) * 4);
            }
          }
          cp_async_wait_all();
          __syncwarp();
        }
      }
      const uint32_t acc_col = b * (BN * MS) + (MS == 2 ? eg * BN : 0);
      for (int c = 0; c < BN / 32; ++c) {
        const int col0 = n0 + c * 32;
        if (col0 >= p.N) break;
        if (MS == 1 && c % C::EPI_GROUPS != eo) continue;
        const float* res_row = nullptr;
        const int rslot = C::RES_G > 0 ? eg * C::RES_G + rcount % C::RES_G : 0;
        if constexpr (RES) {
          if (!warp_wait(&rfull[rslot], (rcount / C::RES_G) & 1, abort_flag, kTimeoutNs)) break;
          res_row = reinterpret_cast<const float*>(sRes + rslot * C::RES_SLOT) + (wq * 32 + lane) * 32;
        }
        if (rows_live) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + acc_col + c * 32 + ((uint32_t)(wq * 32) << 16), r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          const size_t sk_off = sk_wbase + (size_t)c * 4096 + lane;
          if (pc.kind == 1) {
            float* dst = p.sk_ws + (size_t)(unit0 * PAIR + (int)rank) * kSlot + sk_off;
#pragma unroll
            for (int i = 0; i < 32; ++i) __stcg(dst + i * 32, v[i]);
            continue;
          }
          if (pc.kind == 2) {
            const float* stage = reinterpret_cast<const float*>(sA) + (size_t)(warp - 4) * SK_NCAP * SK_MYCH * 1024 +
                                 (MS == 2 ? c : c / C::EPI_GROUPS) * 1024 + lane;
            for (int j = unit0 + 1; j < sk_jfast; ++j) {
              const float* src = stage + (j - unit0 - 1) * SK_MYCH * 1024;
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += src[i * 32];
            }
            for (int j = sk_jfast; j < sk_j1; ++j) {
              const float* src = p.sk_ws + (size_t)(j * PAIR + (int)rank) * kSlot + sk_off;
              float q[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) q[i] = __ldcg(src + i * 32);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += q[i];
            }
          }
          if (!raw) {
            if (!unit_alpha) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] *= p.alpha;
            }
            if (p.bias) {
              // the owned-chunk index c / EPI_GROUPS is a compile-time constant after unrolling
              float bias_lane = bias_reg[0];
#pragma unroll
              for (int i = 1; i < MYCH; ++i)
                if ((MS == 2 ? c : c / C::EPI_GROUPS) == i) bias_lane = bias_reg[i];
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += __shfl_sync(0xffffffffu, bias_lane, i);
            }
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
              for (int i = 0; i < 32; ++i) v[i] = silu_fast(v[i]);
            }
            if (p.round_out) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = to_tf32_rna(v[i]);
            }
          }
          float* st_out =
              reinterpret_cast<float*>(sOut + ((nstore % C::OUT_BUFS) * C::EPI_WARPS + (warp - 4)) * 4096);
          // the store that last used this buffer has read it
          if (lane == 0) tma_store_wait_read<C::OUT_BUFS - 1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            *reinterpret_cast<float4*>(st_out + lane * 32 + ((j ^ (lane & 7)) * 4)) =
                make_float4(v[4 * j + 0], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&mapY, st_out, col0, row0, z);
            tma_store_commit();
          }
          ++nstore;
        }
        if constexpr (RES) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&rempty[rslot]);
          ++rcount;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR == 2)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[b]), 0));
        else
          mbar_arrive(&tempty[b]);
        if (pc.kind == 1) {  // publish this warp's part of the partial
          __threadfence();
          atomicAdd(p.sk_flags + unit0 * PAIR + (int)rank, 1);
        } else if (pc.kind == 2) {  // done with the contributors' slots; the last reader clears
          for (int j = unit0 + 1; j < sk_j1; ++j)
            if (atomicAdd(p.sk_flags + j * PAIR + (int)rank, 1) == 2 * C::EPI_WARPS - 1)
              atomicExch(p.sk_flags + j * PAIR + (int)rank, 0);
        }
      }
    }
    // the stores' shared-memory reads are done before the CTA may exit; their global writes
    // complete with the grid, which is what a dependent launch waits for
    if (lane == 0) tma_store_wait_read0();
    __syncwarp();
  }

  __syncthreads();
  // In a pair, neither CTA leaves while the other may still touch its shared memory or TMEM.
  if constexpr (PAIR == 2) cluster_sync();
  if (warp == 2) {
    tc_fence_after();
    if constexpr (PAIR == 2)
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && p.err) atomicExch(p.err, 1);
}

// Split-K finish: y = epilogue(alpha * sum_k ws[k] + bias (+ residual)), the planes summed in
// index order so that the result does not depend on which CTA finished first.  Four output
// columns per thread; the pad columns of y beyond N are never written.
__global__ void __launch_bounds__(256)
    splitk_finish_kernel(const float* __restrict__ ws, int ksplit, int M, int N, int ldw, float alpha,
                         const float* __restrict__ bias, const float* __restrict__ res, int ldr, int act,
                         int round_out, float* __restrict__ y, int ldy) {
  // launched as a programmatic dependent of the split GEMM: its CTAs may be resident before
  // the partials are complete, and wait here until they are
  griddep_wait();
  griddep_launch_dependents();
  const int groups = (N + 3) >> 2;
  const long total = (long)M * groups;
  const size_t plane = (size_t)M * ldw;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int m = (int)(i / groups);
    const int n = (int)(i - (long)m * groups) * 4;
    const float* src = ws + (size_t)m * ldw + n;
    float4 acc = __ldcs(reinterpret_cast<const float4*>(src));
    for (int k = 1; k < ksplit; ++k) {
      const float4 t = __ldcs(reinterpret_cast<const float4*>(src + k * plane));
      acc.x += t.x;
      acc.y += t.y;
      acc.z += t.z;
      acc.w += t.w;
    }
    float v[4] = {alpha * acc.x, alpha * acc.y, alpha * acc.z, alpha * acc.w};
    if (bias) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] += n + j < N ? __ldg(bias + n + j) : 0.0f;
    }
    if (res) {
      const float4 r = *reinterpret_cast<const float4*>(res + (size_t)m * ldr + n);
      v[0] += r.x;
      v[1] += r.y;
      v[2] += r.z;
      v[3] += r.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (act == 1 || act == 5) v[j] = v[j] < 0.0f ? 0.0f : v[j];
      else if (act == 3) v[j] = silu_fast(v[j]);
      if (round_out) v[j] = round_tf32_bits(v[j]);
    }
    float* dst = y + (size_t)m * ldy + n;
    if (n + 4 <= N) {
      *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      for (int j = 0; j < N - n; ++j) dst[j] = v[j];
    }
  }
}

// Launches overlap the previous kernel's tail (programmatic dependent launch) unless
// SPINN_NO_PDL is set.
bool pdl_enabled() {
  static const bool on = getenv("SPINN_NO_PDL") == nullptr;
  return on;
}

// Co-resident clusters of two CTAs for a pair variant (queried once per variant and device
// by the caller).
template <typename K>
int pair_clusters(K kern, uint32_t smem, int threads, int sms) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = sms / 2;
  }
  return n;
}

template <int BN, int CB, int MODE, bool RES, int PAIR, int BK, int MS = 1, bool WR = false>
int launch_variant(const AMaps& ma, const CUtensorMap& mb, const CUtensorMap& my, const CUtensorMap& mr,
                   const TcParams& p, int sms, cudaStream_t stream) {
  using C = Cfg<BN, CB, RES, PAIR, BK, MS, WR>;
  auto kern = tc_gemm_kernel<BN, CB, MODE, RES, PAIR, BK, MS, WR>;
  if (WR && (p.tiles_n != 1 || (uint32_t)p.num_kb * C::B_STAGE > C::W_BYTES)) {
    set_error("tcgen05 gemm: resident weights need one N tile and at most %u bytes of W", C::W_BYTES);
    return SPINN_CUDA_EINVAL;
  }
  // The opt-in shared-memory size is a per-device function attribute: set it once per device.
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  SPINN_CUDA_TRY(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    SPINN_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    configured.fetch_or(bit);
  }
  TcParams q = p;
  q.nstages = C::STAGES;
  if (const char* e = getenv("SPINN_TC_STAGES")) {  // tuning: use fewer ring stages
    const int v = atoi(e);
    if (v >= 2 && v < C::STAGES) q.nstages = v;
  }
  int grid;
  if constexpr (PAIR == 1)
    grid = (int)std::min<long>(q.num_units, sms);
  else
  {
    static std::atomic<int> clusters[64];
    int nc = clusters[dev & 63].load();
    if (nc <= 0) {
      nc = pair_clusters(kern, C::SMEM, C::THREADS, sms);
      clusters[dev & 63].store(nc);
    }
    grid = 2 * (int)std::min<long>(q.num_units, nc);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (pdl_enabled()) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if constexpr (PAIR == 2) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 2;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  SPINN_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ma, mb, my, mr, q));
  SPINN_CUDA_TRY(cudaGetLastError());
  return 0;
}

template <int MODE, bool RES>
int dispatch_bn_cb(int bn, int cb, int pair, int bk, int ms, int wr, const AMaps& ma, const CUtensorMap& mb,
                   const CUtensorMap& my, const CUtensorMap& mr, const TcParams& p, int sms, cudaStream_t s) {
#define SPINN_TC_CASE(BNV, CBV, PV, BKV)                                             \
  if (bn == BNV && cb == CBV && pair == PV && bk == BKV && ms == 1 && !wr) \
    return launch_variant<BNV, CBV, MODE, RES, PV, BKV>(ma, mb, my, mr, p, sms, s);
#define SPINN_TC_CASE2(BNV, CBV, BKV)                                               \
  if (bn == BNV && cb == CBV && pair == 1 && bk == BKV && ms == 2 && !wr) \
    return launch_variant<BNV, CBV, MODE, RES, 1, BKV, 2>(ma, mb, my, mr, p, sms, s);
#define SPINN_TC_CASE2W(BNV, CBV, BKV)                                             \
  if (bn == BNV && cb == CBV && pair == 1 && bk == BKV && ms == 2 && wr) \
    return launch_variant<BNV, CBV, MODE, RES, 1, BKV, 2, true>(ma, mb, my, mr, p, sms, s);
  SPINN_TC_CASE(256, 32, 1, 32) SPINN_TC_CASE(128, 32, 1, 32) SPINN_TC_CASE(64, 32, 1, 32)
  SPINN_TC_CASE2(128, 32, 32) SPINN_TC_CASE2(64, 32, 32)
  if constexpr (!RES) {
    SPINN_TC_CASE(128, 32, 1, 64) SPINN_TC_CASE(64, 32, 1, 64)
    SPINN_TC_CASE(256, 32, 2, 64) SPINN_TC_CASE(128, 32, 2, 64)
    SPINN_TC_CASE2(128, 32, 64) SPINN_TC_CASE2(64, 32, 64)
    SPINN_TC_CASE2W(64, 32, 32) SPINN_TC_CASE2W(64, 32, 64)
  }
  if constexpr (MODE == kIm2col) {
    SPINN_TC_CASE(256, 16, 1, 32) SPINN_TC_CASE(128, 16, 1, 32) SPINN_TC_CASE(64, 16, 1, 32)
    SPINN_TC_CASE(256, 8, 1, 32) SPINN_TC_CASE(128, 8, 1, 32) SPINN_TC_CASE(64, 8, 1, 32)
    SPINN_TC_CASE(256, 4, 1, 32) SPINN_TC_CASE(128, 4, 1, 32) SPINN_TC_CASE(64, 4, 1, 32)
    SPINN_TC_CASE2(128, 16, 32) SPINN_TC_CASE2(64, 16, 32)
    if constexpr (!RES) {
      SPINN_TC_CASE(128, 16, 1, 64) SPINN_TC_CASE(64, 16, 1, 64)
      SPINN_TC_CASE(256, 16, 2, 64) SPINN_TC_CASE(128, 16, 2, 64)
      SPINN_TC_CASE2(128, 16, 64) SPINN_TC_CASE2(64, 16, 64)
      SPINN_TC_CASE2W(64, 16, 32) SPINN_TC_CASE2W(64, 16, 64)
    }
  }
#undef SPINN_TC_CASE
#undef SPINN_TC_CASE2
#undef SPINN_TC_CASE2W
  set_error("tcgen05 gemm: no variant for BN=%d CB=%d pair=%d BK=%d MS=%d WR=%d mode=%d", bn, cb, pair, bk, ms, wr,
            MODE);
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

// Largest split-K workspace a launch may use.
constexpr size_t kWsCap = size_t(64) << 20;

struct TilePlan {
  int bn = 256;
  int pair = 1;  // 2: CTA pairs with 256-row tiles (cta_group::2)
  int ms = 1;    // 2: one CTA, 256-row tiles as two 128-row sub-tiles
  int wr = 0;    // 1: W resident in shared memory (one N tile, small K)
  int bk = 32;   // K depth of a pipeline stage
  int ksplit = 1;
  int kb_per = 1;
  int sk = 0;  // stream-K schedule over all slots
  size_t ws_bytes = 0;
};

// Optional override for tuning sweeps: SPINN_TC_TILES="bn,ksplit[,pair[,bk[,ms[,wr[,sk]]]]]"
// (read at each launch; a captured graph keeps the choice made when it was captured; wr and
// sk: -1 = no, 1 = yes, 0 = planner's choice).
void forced_tiles(int* bn, int* ks, int* pair, int* bk, int* ms, int* wr, int* sk) {
  *bn = -1;
  *ks = 0;
  *pair = 0;
  *bk = 0;
  *ms = 0;
  *wr = 0;
  *sk = 0;
  const char* e = getenv("SPINN_TC_TILES");
  if (e && sscanf(e, "%d,%d,%d,%d,%d,%d,%d", bn, ks, pair, bk, ms, wr, sk) < 1) *bn = -1;
}

// Chooses the tile shape (BN, single CTA or CTA pair, stage depth) and the K split from a
// cost model fitted to measured B200 layer times at batches 32 and 256 (microseconds,
// ~1.9 GHz; geometric error ~13%).  A launch costs a fixed 14 (launch ramp, pipeline fill,
// the last tile's exposed epilogue) plus 2 per extra wave of work units.  A unit costs the
// larger of its main loop and its epilogue (0.8 per 32 output columns and epilogue warp
// group, overlapped with the next unit's main loop through the other TMEM accumulators).
// Main-loop stages cost about the same whatever their width -- they are bounded by the
// per-stage barrier handoff and the per-box TMA issue cost as much as by tensor throughput --
// so deep stages, CTA pairs (twice the rows per MMA) and two M sub-tiles per CTA (256-row A
// boxes, one W box per two MMAs) pay off.  A split adds the finish pass: (ksplit + 2) x M x N
// floats at 8 TB/s (the partials are L2-resident).  64-deep stages and sub-tiles need channel
// blocks of 16 or 32 and no fused residual (the residual ring would leave too few stages).
//
// Stream-K (allow_sk: a flag buffer is at hand, batch 1) spreads the tiles' k-blocks evenly
// over every slot, so a last wave that would leave slots idle does not: the main loop costs
// ceil(tiles x k-blocks / slots) stages, each ~10% dearer than the fit with every SM loading
// (measured: 0.68 against 0.62 us for 256-wide pairs), plus ~10 us that ResNet-101's 14x14
// and 7x7 layers measured beyond that at batches 64-256 (the head worker's exposed tail: a
// contributor that ends with it, the partial-sum copy, then the epilogue).  So it pays where
// a long reduction leaves a short last wave -- the 512-channel 7x7 3x3 layers at batch 256, 98
// pair tiles on 74 slots: 110 -> 89 us -- and not for short ones.  Only for problems of at
// most four waves of whole tiles: across many waves the tile order of the ordinary schedule
// keeps L2 locality that stream-K ranges lose (the stem and the 56x56 1x1 layers measured
// 10-25% slower), and the last wave matters little there.
TilePlan plan_tiles(int M, int N, int K, int cb, bool has_res, int sms, size_t ws_limit, int force_bn,
                    bool allow_wr, int taps, bool allow_sk) {
  int fbn, fks, fpair, fbk, fms, fwr, fsk;
  forced_tiles(&fbn, &fks, &fpair, &fbk, &fms, &fwr, &fsk);
  if (fsk < 0 || fks > 1 || has_res || sms > kTcSkFlags) allow_sk = false;
  if (force_bn <= 0 && (fbn == 64 || fbn == 128 || fbn == 256)) force_bn = fbn;
  struct Shape {
    int bn, pair, bk, ms, wr;
    double per_stage;
  };
  // Resident-weight shapes come first: when the epilogue term dominates a narrow tile both
  // kinds cost the same in the model, and the measured stems favour resident weights
  // (the 3->16-channel 640x640 stem at batch 32: 121 vs 199 us).
  const Shape shapes[13] = {{64, 1, 64, 2, 1, 0.45},   {64, 1, 32, 2, 1, 0.25},   {256, 1, 32, 1, 0, 0.332},
                            {128, 1, 32, 1, 0, 0.266}, {64, 1, 32, 1, 0, 0.237},  {128, 1, 64, 1, 0, 0.405},
                            {64, 1, 64, 1, 0, 0.319},  {256, 2, 64, 1, 0, 0.617}, {128, 2, 64, 1, 0, 0.456},
                            {128, 1, 32, 2, 0, 0.46},  {64, 1, 32, 2, 0, 0.38},   {128, 1, 64, 2, 0, 0.86},
                            {64, 1, 64, 2, 0, 0.67}};
  const size_t ldw = (size_t)((N + 3) & ~3);
  // Multi-tap im2col problems (3x3 and larger filters) load A one tap box per channel block;
  // for 128-row single-CTA tiles with 64-deep stages that costs ~1.3x the stage time of the
  // fit (forced-tile sweep of ResNet-101's 3x3 layers at batch 256: 0.57-0.60 us per stage
  // against 0.405), while the pair and two-sub-tile shapes matched it.
  const double im2col_single64 = taps > 1 ? 1.3 : 1.0;
  TilePlan best, best_sk;
  double best_cost = 1e300, best_sk_cost = 1e300;
  long best_waves = 0;
  for (const Shape& sh : shapes) {
    const int bn = sh.bn;
    if (force_bn > 0 && bn != force_bn) continue;
    if (fpair > 0 && sh.pair != fpair) continue;
    if (fbk > 0 && sh.bk != fbk) continue;
    if (fms > 0 && sh.ms != fms) continue;
    if ((fwr > 0 && !sh.wr) || (fwr < 0 && sh.wr)) continue;
    // resident weights: one N tile, all of W within the resident region, no residual
    if (sh.wr && (!allow_wr || has_res || N > sh.bn || (cb != 32 && cb != 16) ||
                  (size_t)((K + sh.bk - 1) / sh.bk) * sh.bn * sh.bk * 4 > kWresBytes))
      continue;
    if (sh.bk == 64 && ((cb != 32 && cb != 16) || has_res)) continue;
    // sub-tiles with a fused residual: correct (forced shapes) but measured no faster than
    // 256-wide single tiles, and the model cannot tell them apart, so not chosen by default
    if (sh.ms == 2 && ((cb != 32 && cb != 16) || (has_res && (sh.bk != 32 || fms != 2)))) continue;
    if (force_bn <= 0 && sh.pair == 1 && bn > 64 && bn >= 2 * ((N + 63) / 64) * 64) continue;  // far wider than N
    const int slots = sh.pair == 2 ? sms / 2 : sms;
    const double per_stage = sh.per_stage * (sh.pair == 1 && sh.ms == 1 && sh.bk == 64 ? im2col_single64 : 1.0);
    const int num_kb = (K + sh.bk - 1) / sh.bk;
    const int tm = kBM * sh.pair * sh.ms;
    const long tiles = (long)((M + tm - 1) / tm) * ((N + bn - 1) / bn);
    const double epi1 = sh.ms == 2 ? 0.8 * (bn / 32) : 0.8 * (bn / 32) / ((has_res && bn == 256) ? 1 : 2);
    const long total_kb = tiles * num_kb;
    const size_t sk_ws = (size_t)sms * kBM * sh.ms * bn * 4;  // one slot per CTA
    if (allow_sk && !sh.wr && total_kb >= 2L * slots && sk_ws <= ws_limit) {
      const long per = (total_kb + slots - 1) / slots;  // k-blocks per worker
      const long pieces = (per + num_kb - 1) / num_kb + 1;
      const double parts = per >= num_kb ? 1.0 : (double)((num_kb + per - 1) / per);
      const double cost = 14.0 + std::max(per * per_stage * 1.1, pieces * epi1) + 9.0 + parts * (bn * sh.ms / 256.0);
      if (cost < best_sk_cost - 1e-9) {
        best_sk_cost = cost;
        best_sk.bn = bn;
        best_sk.pair = sh.pair;
        best_sk.bk = sh.bk;
        best_sk.ms = sh.ms;
        best_sk.wr = 0;
        best_sk.ksplit = 1;
        best_sk.kb_per = num_kb;
        best_sk.sk = 1;
        best_sk.ws_bytes = sk_ws;
      }
    }
    for (int ks = 1; ks <= 32; ++ks) {
      const int kb_per = (num_kb + ks - 1) / ks;
      const int kse = (num_kb + kb_per - 1) / kb_per;  // slices actually used
      if (kse != ks) continue;
      if (fks > 0 && ks != fks) continue;
      if (ks > 1 && kb_per * sh.bk < 128 && fks <= 0) break;
      const size_t ws = ks > 1 ? (size_t)ks * M * ldw * 4 : 0;
      if (ws > ws_limit) break;
      const long units = tiles * ks;
      const long waves = (units + slots - 1) / slots;
      // epilogue: ~0.8 us per 32-column chunk and warp group; 256-wide residual tiles use one
      // group; with two M sub-tiles each group drains a whole sub-tile
      const double epi = epi1;
      double cost = 14.0 + (waves - 1) * 2.0 + waves * std::max(kb_per * per_stage, epi);
      if (ks > 1) cost += (double)(ks + 2) * M * N * 4 / 8.0e6;
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best_waves = waves;
        best.bn = bn;
        best.pair = sh.pair;
        best.bk = sh.bk;
        best.ms = sh.ms;
        best.wr = sh.wr;
        best.ksplit = ks;
        best.kb_per = kb_per;
        best.ws_bytes = ws;
      }
    }
  }
  if (best_sk_cost < 1e300 && (fsk > 0 || (best_waves <= 4 && best_sk_cost < best_cost - 1.0))) return best_sk;
  if (best_cost == 1e300) {  // forced shape infeasible: single-CTA tiles of the forced width, no split
    best.bn = force_bn > 0 ? force_bn : 256;
    best.pair = 1;
    best.bk = 32;
    best.ms = 1;
    best.wr = 0;
    best.ksplit = 1;
    best.kb_per = (K + 31) / 32;
    best.ws_bytes = 0;
  }
  return best;
}

int problem_k(const TcGemmArgs& a) { return a.a_mode == 0 ? a.kh * a.kw * a.cpad : a.K; }
int problem_cb(const TcGemmArgs& a) { return a.a_mode == 0 ? channel_block(a.cpad) : 32; }

}  // namespace

size_t tc_gemm_workspace_bytes(const TcGemmArgs& a) {
  if (!tc_gemm_supported(a, nullptr) || a.batch > 1) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return plan_tiles(a.M, a.N, problem_k(a), problem_cb(a), a.res != nullptr, sm_count(dev), kWsCap, a.bn, true,
                    a.a_mode == 0 ? a.kh * a.kw : 1, a.sk != 0)
      .ws_bytes;
}

bool tc_gemm_supported(const TcGemmArgs& a, std::string* why) {
  auto fail = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (a.N <= 0 || a.M <= 0) return fail("empty problem");
  if (a.batch < 1) return fail("batch must be at least 1");
  if (a.batch > 1 && (a.a_mode != 1 || a.res)) return fail("batched GEMM needs a row-major A and no residual");
  if (a.ldy % 4 != 0 || a.ldy < a.N) return fail("output row stride must be a multiple of 4 floats");
  if (a.nparts > 1) {
    // A as the channel concatenation of parts: each a whole number of channel blocks
    if (a.nparts > kMaxAParts || a.batch != 1) return fail("at most four parts of A, no batch");
    const int cb = a.a_mode == 0 ? channel_block(a.cpad) : 32;
    int c = 0;
    for (int i = 0; i < a.nparts; ++i) {
      if (!a.xpart[i] || (reinterpret_cast<uintptr_t>(a.xpart[i]) & 15)) return fail("part of A not 16-byte aligned");
      if (a.part_c0[i] != c || cb == 0 || a.part_cpad[i] % cb) return fail("parts of A are not whole channel blocks");
      c += a.part_cpad[i];
    }
    if (c != (a.a_mode == 0 ? a.cpad : a.K)) return fail("parts of A do not add up to its channels");
  } else if (reinterpret_cast<uintptr_t>(a.x) & 15) {
    return fail("operand not 16-byte aligned");
  }
  if ((reinterpret_cast<uintptr_t>(a.y) & 15) || (reinterpret_cast<uintptr_t>(a.wt) & 15))
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

int launch_flag_wait_selftest(int* err, uint64_t timeout_ns, cudaStream_t s) {
  SPINN_CHECK_ARG(err != nullptr && timeout_ns > 0 && timeout_ns <= 1000000000ull,
                  "flag wait self-test: timeout %llu ns outside (0, 1 s]", (unsigned long long)timeout_ns);
  flag_wait_expiry_kernel<<<1, 32, 0, s>>>(err, (unsigned long long)timeout_ns);
  SPINN_CUDA_TRY(cudaGetLastError());
  return 0;
}

static std::atomic<uint64_t> g_streamk_launches{0};
uint64_t tc_gemm_streamk_launches() { return g_streamk_launches.load(); }

void tc_gemm_plan_for(int M, int N, int K, int cb, bool has_res, int sms, int taps, bool allow_sk, int out[7]) {
  const TilePlan tp = plan_tiles(M, N, K, cb, has_res, sms, kWsCap, 0, true, taps, allow_sk);
  out[0] = tp.bn;
  out[1] = tp.pair;
  out[2] = tp.bk;
  out[3] = tp.ms;
  out[4] = tp.wr;
  out[5] = tp.ksplit;
  out[6] = tp.sk;
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
  const int cb = problem_cb(a);
  const int K = problem_k(a);
  if (tc_num_kb(K) * 32 > a.kpad) {
    set_error("tcgen05 gemm: weights padded to %d, need %d", a.kpad, tc_num_kb(K) * 32);
    return SPINN_CUDA_EINVAL;
  }
  const size_t ws_limit = (a.ws && a.batch == 1) ? std::min(a.ws_bytes, kWsCap) : 0;  // batched: no split
  const TilePlan tp = plan_tiles(a.M, a.N, K, cb, a.res != nullptr, sms, ws_limit, a.bn, a.batch == 1,
                                 a.a_mode == 0 ? a.kh * a.kw : 1, a.sk && a.sk_flags && a.batch == 1);
  const int arows = kBM * tp.ms;  // A rows per box
  AMaps ma;
  CUtensorMap mb, my, mr;
  int rc;
  const int nparts = a.nparts > 1 ? a.nparts : 1;
  p.nparts = nparts;
  for (int i = 0; i < kMaxAParts; ++i) p.part_c0[i] = i < nparts && a.nparts > 1 ? a.part_c0[i] : 0;
  if (a.a_mode == 0) {
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
    for (int i = 0; i < nparts; ++i) {
      const float* x = nparts > 1 ? a.xpart[i] : a.x;
      const int c = nparts > 1 ? a.part_cpad[i] : a.cpad;
      rc = encode_im2col_4d(&ma.m[i], x, a.n, a.h, a.w, c, lw, lh, uw, uh, cb, arows, a.sw, a.sh, swizzle_for(cb));
      if (rc) return rc;
    }
  } else {
    p.cpad = a.K;
    p.taps = 1;
    p.kw = 1;
    for (int i = 0; i < nparts; ++i) {
      const float* x = nparts > 1 ? a.xpart[i] : a.x;
      const int k = nparts > 1 ? a.part_cpad[i] : a.K, ld = nparts > 1 ? a.part_cpad[i] : a.lda;
      rc = encode_tiled_3d(&ma.m[i], x, (uint64_t)k, (uint64_t)a.M, (uint64_t)a.batch, (uint64_t)ld * 4, 32,
                           (uint32_t)arows, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
  }
  p.num_kb = (K + tp.bk - 1) / tp.bk;  // stages beyond kpad read zero weights
  const int bn = tp.bn;
  const bool split = tp.ksplit > 1;
  rc = encode_tiled_3d(&mb, a.wt, (uint64_t)a.kpad, (uint64_t)a.N, (uint64_t)(a.b_batched ? a.batch : 1),
                       (uint64_t)a.kpad * 4, (uint32_t)cb, (uint32_t)(bn / tp.pair), swizzle_for(cb));
  if (rc) return rc;
  const int ldw = (a.N + 3) & ~3;
  rc = split ? encode_tiled_3d(&my, a.ws, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)tp.ksplit, (uint64_t)ldw * 4, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_128B)
             : encode_tiled_3d(&my, a.y, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.batch, (uint64_t)a.ldy * 4, 32,
                               32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (a.res && !split) {
    rc = encode_tiled_2d(&mr, a.res, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.ldr * 4, 32, kBM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    mr = my;
  }
  p.tiles_n = (a.N + bn - 1) / bn;
  const int tm = kBM * tp.pair * tp.ms;
  const long tiles = (long)((a.M + tm - 1) / tm) * p.tiles_n;
  if (tiles > 0x7FFFFFFF) {
    set_error("tcgen05 gemm: too many tiles");
    return SPINN_CUDA_EINVAL;
  }
  p.num_tiles = (int)tiles;
  p.ksplit = tp.ksplit;
  p.kb_per = split ? tp.kb_per : p.num_kb;
  p.batch = a.batch;
  p.b_batched = a.b_batched;
  p.reverse = a.reverse;
  const long zs = a.batch > 1 ? a.batch : tp.ksplit;
  if (tiles * zs > 0x7FFFFFFF) {
    set_error("tcgen05 gemm: too many work units");
    return SPINN_CUDA_EINVAL;
  }
  p.num_units = (int)(tiles * zs);
  if (tp.sk) {
    // every slot is a worker (the grid is min(num_units, slots)); each gets >= 2 k-blocks
    const long total = tiles * p.num_kb;
    if (total > 0x7FFFFFFF) {
      set_error("tcgen05 gemm: too many k-blocks for stream-K");
      return SPINN_CUDA_EINVAL;
    }
    p.num_units = (int)total;
    p.sk = 1;
    p.sk_ws = a.ws;
    p.sk_flags = a.sk_flags;
    g_streamk_launches.fetch_add(1);
  }

  p.has_res = a.res != nullptr && !split;
  p.act = a.act;
  p.round_out = a.round_out;
  p.alpha = a.alpha;
  p.bias = a.bias;
  p.err = a.err ? a.err : device_error_flag(dev);
  const int pr = tp.pair, ms = tp.ms, wr = tp.wr;
  if (a.a_mode == 0)
    rc = p.has_res ? dispatch_bn_cb<kIm2col, true>(bn, cb, pr, tp.bk, ms, wr, ma, mb, my, mr, p, sms, stream)
                   : dispatch_bn_cb<kIm2col, false>(bn, cb, pr, tp.bk, ms, wr, ma, mb, my, mr, p, sms, stream);
  else
    rc = p.has_res ? dispatch_bn_cb<kTiled, true>(bn, cb, pr, tp.bk, ms, wr, ma, mb, my, mr, p, sms, stream)
                   : dispatch_bn_cb<kTiled, false>(bn, cb, pr, tp.bk, ms, wr, ma, mb, my, mr, p, sms, stream);
  if (rc || !split) return rc;
  const long groups = (long)a.M * ((a.N + 3) / 4);
  const int fgrid = (int)std::min<long>((groups + 255) / 256, (long)sms * 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(fgrid, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  SPINN_CUDA_TRY(cudaLaunchKernelEx(&cfg, splitk_finish_kernel, (const float*)a.ws, tp.ksplit, a.M, a.N, ldw, a.alpha,
                                    a.bias, a.res, a.ldr, a.act, a.round_out, a.y, a.ldy));
  SPINN_CUDA_TRY(cudaGetLastError());
  return 0;
}

}  // namespace spinn
