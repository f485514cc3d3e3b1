// glue.cu -- memory-bound kernels around the tensor-core path: NCHW<->NHWC layout
// conversion, pooling, elementwise operators, depthwise / grouped direct convolution,
// transposes.  All of them are HBM-bound; they move 16-byte vectors along the contiguous
// channel dimension of NHWC tensors and size grids to fill every SM.
//
// Semantics follow the reference operators cited at each kernel; layouts are NHWC with the
// channel dimension padded to `cpad` (a multiple of 4) where the tensor-core path needs it.
#include <algorithm>
#include <atomic>

#include "internal.h"
#include "ptx.cuh"

namespace spinn {

namespace {

constexpr int kEltThreads = 256;

inline int grid_for(long work, int threads, int max_blocks = 148 * 32) {
  long b = (work + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return (int)b;
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == 1 || act == 5) return v < 0.0f ? 0.0f : v;
  if (act == 3) return silu_fast(v);
  return v;
}

// [n][c][hw] -> [n][hw][cpad] through a 32x33 shared tile; channels >= c are written as 0.
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, int c, int hw, int cpad,
                                    int round_tf32) {
  __shared__ float tile[32][33];
  const int n = blockIdx.z;
  const int hw0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* xn = x + (size_t)n * c * hw;
  float* yn = y + (size_t)n * hw * cpad;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int cc = c0 + i, p = hw0 + threadIdx.x;
    tile[i][threadIdx.x] = (cc < c && p < hw) ? xn[(size_t)cc * hw + p] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int p = hw0 + i, cc = c0 + threadIdx.x;
    if (p < hw && cc < cpad) {
      const float v = tile[threadIdx.x][i];
      yn[(size_t)p * cpad + cc] = round_tf32 ? to_tf32_rna(v) : v;
    }
  }
}

__global__ void nhwc_to_nchw_kernel(const float* __restrict__ x, float* __restrict__ y, int c, int hw, int cpad) {
  __shared__ float tile[32][33];
  const int n = blockIdx.z;
  const int hw0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* xn = x + (size_t)n * hw * cpad;
  float* yn = y + (size_t)n * c * hw;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int p = hw0 + i, cc = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (p < hw && cc < c) ? xn[(size_t)p * cpad + cc] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int cc = c0 + i, p = hw0 + threadIdx.x;
    if (cc < c && p < hw) yn[(size_t)cc * hw + p] = tile[threadIdx.x][i];
  }
}

// One thread per output pixel (b, i, j): 16 channels = 4 phases (dy, dx) x 4 input channels.
template <typename Idx>
__global__ void space_to_depth2_kernel(const float* __restrict__ x, float4* __restrict__ y, int n, int c, int h,
                                       int w, int h2, int w2, int ph, int pw, int round_tf32) {
  const Idx total = (Idx)n * h2 * w2;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const int j = (int)(i % w2);
    Idx t = i / w2;
    const int r = (int)(t % h2);
    const int b = (int)(t / h2);
#pragma unroll
    for (int ph4 = 0; ph4 < 4; ++ph4) {
      const int iy = 2 * r + (ph4 >> 1) - ph, ix = 2 * j + (ph4 & 1) - pw;
      const bool in = iy >= 0 && iy < h && ix >= 0 && ix < w;
      float v[4];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch)
        v[ch] = (in && ch < c) ? __ldg(x + (((size_t)b * c + ch) * h + iy) * w + ix) : 0.0f;
      if (round_tf32) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) v[ch] = to_tf32_rna(v[ch]);
      }
      y[i * 4 + ph4] = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}

// MaxPool (SPINN/run_time/ops/pool/maxpool.c:5-49): -1e30 start, padded taps skipped.
template <typename Idx>
__global__ void maxpool_nhwc_kernel(const float4* __restrict__ x, float4* __restrict__ y, int n, int h, int w,
                                    int c4, int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw) {
  // Idx = int when the element count fits: 64-bit division would dominate this HBM-bound loop.
  const Idx total = (Idx)n * oh * ow * c4;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const int cq = (int)(i % c4);
    Idx t = i / c4;
    const int ox = (int)(t % ow);
    t /= ow;
    const int oy = (int)(t % oh);
    const int b = (int)(t / oh);
    float4 m = make_float4(-1e30f, -1e30f, -1e30f, -1e30f);  // the reference's initial value (maxpool.c:32)
    for (int r = 0; r < kh; ++r) {
      const int iy = oy * sh - ph + r;
      if (iy < 0 || iy >= h) continue;
      for (int s = 0; s < kw; ++s) {
        const int ix = ox * sw - pw + s;
        if (ix < 0 || ix >= w) continue;
        const float4 v = __ldg(x + (((size_t)b * h + iy) * w + ix) * c4 + cq);
        m.x = v.x > m.x ? v.x : m.x;
        m.y = v.y > m.y ? v.y : m.y;
        m.z = v.z > m.z ? v.z : m.z;
        m.w = v.w > m.w ? v.w : m.w;
      }
    }
    y[i] = m;
  }
}

// MaxPool 3x3 stride 2 (the ResNet stem pool), one CTA per TY x TX output pixels of one image:
// the (2 TY + 1) x (2 TX + 1) input window of all channels is read once with coalesced float4
// loads into shared memory (taps outside the image read as -1e30, which a max over taps that
// includes a real one ignores, as the reference skips them), then each output takes its nine
// taps from there.  Nine global loads per output become ~1.2.
constexpr int kPoolTY = 4, kPoolTX = 8, kPoolThreads = 256, kPoolMaxC4 = 16;
__global__ void __launch_bounds__(kPoolThreads) maxpool3s2_tile_kernel(const float4* __restrict__ x,
                                                                      float4* __restrict__ y, int h, int w, int c4,
                                                                      int oh, int ow, int ph, int pw) {
  constexpr int IH = 2 * kPoolTY + 1, IW = 2 * kPoolTX + 1;
  __shared__ float4 tile[IH * IW * kPoolMaxC4];
  const int ox0 = blockIdx.x * kPoolTX, oy0 = blockIdx.y * kPoolTY, b = blockIdx.z;
  const int iy0 = 2 * oy0 - ph, ix0 = 2 * ox0 - pw;
  const float4* xb = x + (size_t)b * h * w * c4;
  const int nin = IH * IW * c4;
  // all of this thread's loads issued before the first store, so they are in flight together
  constexpr int PER = (IH * IW * kPoolMaxC4 + kPoolThreads - 1) / kPoolThreads;
  float4 v[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int e = threadIdx.x + k * kPoolThreads;
    const int cq = e % c4, px = e / c4, col = px % IW, r = px / IW;
    const int iy = iy0 + r, ix = ix0 + col;
    v[k] = (e < nin && iy >= 0 && iy < h && ix >= 0 && ix < w) ? __ldg(xb + ((size_t)iy * w + ix) * c4 + cq)
                                                              : make_float4(-1e30f, -1e30f, -1e30f, -1e30f);
  }
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int e = threadIdx.x + k * kPoolThreads;
    if (e < nin) tile[e] = v[k];
  }
  __syncthreads();
  const int nout = kPoolTY * kPoolTX * c4;
  for (int e = threadIdx.x; e < nout; e += kPoolThreads) {
    const int cq = e % c4, px = e / c4, tx = px % kPoolTX, ty = px / kPoolTX;
    const int oy = oy0 + ty, ox = ox0 + tx;
    if (oy >= oh || ox >= ow) continue;
    float4 m = make_float4(-1e30f, -1e30f, -1e30f, -1e30f);  // the reference's initial value (maxpool.c:32)
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        const float4 v = tile[((2 * ty + r) * IW + 2 * tx + s) * c4 + cq];
        m.x = v.x > m.x ? v.x : m.x;
        m.y = v.y > m.y ? v.y : m.y;
        m.z = v.z > m.z ? v.z : m.z;
        m.w = v.w > m.w ? v.w : m.w;
      }
    y[(((size_t)b * oh + oy) * ow + ox) * c4 + cq] = m;
  }
}

// Self-test of the bounded-wait path every tcgen05 kernel relies on: one thread waits on an
// mbarrier that nothing arrives at, with the same mbar_wait the GEMM uses, gives up after
// `timeout_ns` and raises the device error flag (code 2).  Nothing faults or hangs.
__global__ void wait_expiry_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0, &abort_flag, timeout_ns)) atomicExch(err, 2);
}

// TopK (SPINN/run_time/ops/tensor/topk.c:20-87): for every row of the last axis, the k largest
// values in descending order and their int64 indices.  One CTA sorts a row in shared memory
// (bitonic network over 64-bit keys: order-preserving bits of the value, inverted, above the
// index), so equal values come out in ascending index order -- the order the reference's
// qsort (glibc merge sort, a stable sort for its comparator) produces.  -0.0 and +0.0 share a
// key, as they compare equal there; values are copied from the row itself.
__global__ void __launch_bounds__(1024) topk_rows_kernel(const float* __restrict__ x, int n, int k, int npow2,
                                                         float* __restrict__ vals, int64_t* __restrict__ idx) {
  extern __shared__ unsigned long long keys[];
  const float* row = x + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
    unsigned long long key = ~0ull;  // padding sorts last
    if (i < n) {
      uint32_t u = __float_as_uint(row[i]);
      if (u == 0x80000000u) u = 0;  // -0.0 == +0.0
      const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // increases with the value
      key = ((unsigned long long)(~ord) << 32) | (uint32_t)i;
    }
    keys[i] = key;
  }
  __syncthreads();
  for (int size = 2; size <= npow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < npow2 / 2; t += blockDim.x) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool ascending = (lo & size) == 0;
        const unsigned long long a = keys[lo], b = keys[hi];
        if ((a > b) == ascending) {
          keys[lo] = b;
          keys[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const uint32_t j = (uint32_t)keys[i];
    vals[(size_t)blockIdx.x * k + i] = row[j];
    idx[(size_t)blockIdx.x * k + i] = (int64_t)j;
  }
}

// Row-strided copy for Concat/Split (SPINN/run_time/ops/tensor/concat.c, split.c): row r of
// dst gets src's first `width` values and zeros up to `fill_to`.  V = 4: float4 accesses
// (pointers, pitches and both widths multiples of 4 floats).
template <int V, typename Idx>
__global__ void copy_rows_kernel(const float* __restrict__ src, int src_ld, float* __restrict__ dst, int dst_ld,
                                 Idx rows, int width, int fill_to) {
  const int q = fill_to / V;
  const Idx total = rows * q;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const Idx r = i / q;
    const int c = (int)(i - r * q) * V;
    if constexpr (V == 4) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < width) v = __ldg(reinterpret_cast<const float4*>(src + (size_t)r * src_ld + c));
      *reinterpret_cast<float4*>(dst + (size_t)r * dst_ld + c) = v;
    } else {
      dst[(size_t)r * dst_ld + c] = c < width ? __ldg(src + (size_t)r * src_ld + c) : 0.0f;
    }
  }
}

// Concat of up to kCatMaxParts parts along the last (row-contiguous) axis in one launch: one
// thread per float4 of a destination row finds its part by offset; the destination's pad lanes
// past the last part are written as zeros.  Offsets and widths are multiples of 4 floats.
template <typename Idx>
__global__ void concat_rows_kernel(CatParts parts, float* __restrict__ dst, int dst_ld, Idx rows, int fill_to) {
  const int q = fill_to / 4;
  const Idx total = rows * q;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const Idx r = i / q;
    const int c = (int)(i - r * q) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < kCatMaxParts; ++k) {
      if (k < parts.n && c >= parts.off[k] && c < parts.off[k] + parts.width[k])
        v = __ldg(reinterpret_cast<const float4*>(parts.src[k] + (size_t)r * parts.ld[k] + (c - parts.off[k])));
    }
    *reinterpret_cast<float4*>(dst + (size_t)r * dst_ld + c) = v;
  }
}

// The inverse: one thread per float4 of a source row writes it to the part that owns it.
template <typename Idx>
__global__ void split_rows_kernel(SplitParts parts, const float* __restrict__ src, int src_ld, Idx rows, int width) {
  const int q = width / 4;
  const Idx total = rows * q;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const Idx r = i / q;
    const int c = (int)(i - r * q) * 4;
    const float4 v = __ldg(reinterpret_cast<const float4*>(src + (size_t)r * src_ld + c));
#pragma unroll
    for (int k = 0; k < kCatMaxParts; ++k) {
      if (k < parts.n && c >= parts.off[k] && c < parts.off[k] + parts.width[k])
        *reinterpret_cast<float4*>(parts.dst[k] + (size_t)r * parts.ld[k] + (c - parts.off[k])) = v;
    }
  }
}

// Last-axis Concat gathered from pieces (launch_gather_rows): one tile of 32 channels x 128
// positions of one image of one piece per block iteration, staged in shared memory so that
// both the read (along channels for NHWC pieces, along positions for row pieces) and the write
// (along positions) are coalesced; every thread has 16 loads in flight per tile, and the next
// tile's loads are issued before the current one is written.  Tiles run channel tile fastest,
// so blocks working at the same time read all channel slices of the same pixels.  tile0[k] is
// the first tile of piece k.
constexpr int kGatherTL = 128;  // positions per tile
struct GatherTiles {
  long tile0[kGatherMaxPieces + 1];
  int ctiles[kGatherMaxPieces], ltiles[kGatherMaxPieces];
};
__global__ void __launch_bounds__(256) gather_rows_kernel(GatherPieces g, GatherTiles t, float* __restrict__ dst,
                                                          int n, int ctot, int ltot) {
  __shared__ float tile[32][kGatherTL + 1];
  constexpr int V = kGatherTL * 32 / 256;  // values per thread and tile
  const long total = t.tile0[g.n];
  // One tile's parameters, read from the (dynamically indexed) piece table once per tile; the
  // element loops then index with 32-bit offsets from per-tile base pointers (the launcher
  // bounds one image of a piece and one destination row block below 2^31 elements).
  struct Tile {
    const float* src;  // first element this thread's lane column / row reads
    float* dst;        // destination element (channel cb, position lb) of the tile
    int nhwc, ld, cl, ll;  // channels / positions of the tile still inside the piece
  };
  auto tile_of = [&](long u) {
    int k = 0;
    while (k + 1 < g.n && u >= t.tile0[k + 1]) ++k;
    const int local = (int)(u - t.tile0[k]);
    const int per_img = t.ctiles[k] * t.ltiles[k];
    const int b = local / per_img;
    const int r = local - b * per_img;
    const int cb = (r % t.ctiles[k]) * 32, lb = (r / t.ctiles[k]) * kGatherTL;
    Tile x;
    x.nhwc = g.nhwc[k];
    x.ld = g.ld[k];
    x.cl = g.chans[k] - cb;
    x.ll = g.len[k] - lb;
    x.src = g.nhwc[k] ? g.src[k] + (size_t)b * g.len[k] * x.ld + (size_t)lb * x.ld + g.c0[k] + cb
                      : g.src[k] + (size_t)b * g.chans[k] * x.ld + (size_t)cb * x.ld + lb;
    x.dst = dst + ((size_t)b * ctot + g.dst_c[k] + cb) * ltot + g.dst_l[k] + lb;
    return x;
  };
  // value v of a thread: NHWC pieces position ty + 8 v, lane = channel; row pieces channel
  // ty + 8 (v / 4), position (v % 4) * 32 + lane
  auto load = [&](const Tile& x, float (&r)[V]) {
    if (x.nhwc) {
      const bool cin = (int)threadIdx.x < x.cl;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int l = threadIdx.y + 8 * v;
        r[v] = (cin && l < x.ll) ? __ldg(x.src + l * x.ld + threadIdx.x) : 0.0f;
      }
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int c = threadIdx.y + 8 * (v / 4), l = (v % 4) * 32 + threadIdx.x;
        r[v] = (c < x.cl && l < x.ll) ? __ldg(x.src + c * x.ld + l) : 0.0f;
      }
    }
  };
  float r[V];
  long u = blockIdx.x;
  Tile cur{};
  if (u < total) {
    cur = tile_of(u);
    load(cur, r);
  }
  for (; u < total; u += gridDim.x) {
    if (cur.nhwc) {
#pragma unroll
      for (int v = 0; v < V; ++v) tile[threadIdx.x][threadIdx.y + 8 * v] = r[v];
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v) tile[threadIdx.y + 8 * (v / 4)][(v % 4) * 32 + threadIdx.x] = r[v];
    }
    __syncthreads();
    const Tile w = cur;
    const long nu = u + gridDim.x;
    if (nu < total) {  // the next tile's loads are in flight while this one is written
      cur = tile_of(nu);
      load(cur, r);
    }
#pragma unroll
    for (int i = threadIdx.y; i < 32; i += 8)
#pragma unroll
      for (int q = 0; q < kGatherTL / 32; ++q) {
        const int l = q * 32 + threadIdx.x;
        if (i < w.cl && l < w.ll) w.dst[i * ltot + l] = tile[i][l];
      }
    __syncthreads();  // the tile is refilled by the next iteration
  }
}

// AveragePool (SPINN/run_time/ops/pool/avgpool.c): divisor = window taps inside the image,
// or the full window when count_include_pad.
__global__ void avgpool_nhwc_kernel(const float4* __restrict__ x, float4* __restrict__ y, int n, int h, int w,
                                    int c4, int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw,
                                    int include_pad) {
  const long total = (long)n * oh * ow * c4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int cq = (int)(i % c4);
    long t = i / c4;
    const int ox = (int)(t % ow);
    t /= ow;
    const int oy = (int)(t % oh);
    const int b = (int)(t / oh);
    float4 acc = make_float4(0, 0, 0, 0);
    int cnt = 0;
    for (int r = 0; r < kh; ++r) {
      const int iy = oy * sh - ph + r;
      for (int s = 0; s < kw; ++s) {
        const int ix = ox * sw - pw + s;
        if (iy < 0 || iy >= h || ix < 0 || ix >= w) continue;
        const float4 v = x[(((size_t)b * h + iy) * w + ix) * c4 + cq];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
        ++cnt;
      }
    }
    const float d = include_pad ? (float)(kh * kw) : (float)(cnt > 0 ? cnt : 1);
    y[i] = make_float4(acc.x / d, acc.y / d, acc.z / d, acc.w / d);
  }
}

// GlobalAveragePool (SPINN/run_time/ops/pool/global_avg_pool.c:4-28): sequential fp32 sum
// over the spatial positions in order, then one division -- the reference's exact order.
__global__ void gap_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, int n, int hw, int cpad,
                                int round_tf32) {
  const long total = (long)n * cpad;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i % cpad);
    const long b = i / cpad;
    const float* p = x + (size_t)b * hw * cpad + c;
    float s = 0.0f;
    for (int k = 0; k < hw; ++k) s += p[(size_t)k * cpad];
    const float v = s / (float)hw;
    y[i] = round_tf32 ? to_tf32_rna(v) : v;
  }
}

__global__ void binary_kernel(const float* __restrict__ a, long na, const float* __restrict__ b, long nb,
                              float* __restrict__ y, long n, int op, int act) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float u = a[na == n ? i : i % na], v = b[nb == n ? i : i % nb];
    float r;
    switch (op) {
      case ELT_MUL: r = u * v; break;
      case ELT_SUB: r = u - v; break;
      case ELT_DIV: r = u / v; break;
      default: r = u + v; break;
    }
    y[i] = act ? (r < 0.0f ? 0.0f : r) : r;
  }
}

// Same-shape operands (no broadcast), 16-byte aligned, n a multiple of 4: four elements per
// thread with 16-byte accesses; the same arithmetic per element as binary_kernel.
__global__ void binary4_kernel(const float4* __restrict__ a, const float4* __restrict__ b, float4* __restrict__ y,
                               long n4, int op, int act) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 u = a[i], v = b[i];
    float r[4] = {u.x, u.y, u.z, u.w};
    const float w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      switch (op) {
        case ELT_MUL: r[k] = r[k] * w[k]; break;
        case ELT_SUB: r[k] = r[k] - w[k]; break;
        case ELT_DIV: r[k] = r[k] / w[k]; break;
        default: r[k] = r[k] + w[k]; break;
      }
      if (act) r[k] = r[k] < 0.0f ? 0.0f : r[k];
    }
    y[i] = make_float4(r[0], r[1], r[2], r[3]);
  }
}

__global__ void unary_kernel(const float* __restrict__ x, float* __restrict__ y, long n, int op) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = x[i];
    float r;
    switch (op) {
      case UN_RELU: r = v > 0.0f ? v : 0.0f; break;
      case UN_SIGMOID: r = 1.0f / (1.0f + expf(-v)); break;
      case UN_SILU: r = silu_fast(v); break;
      default: r = v; break;
    }
    y[i] = r;
  }
}

// op_batch_norm (SPINN/run_time/ops/norm/batch_norm.c:17-76) with precomputed scale/shift.
__global__ void channel_affine_kernel(const float* __restrict__ x, float* __restrict__ y, long pixels, int cpad,
                                      const float* __restrict__ scale, const float* __restrict__ shift) {
  const long total = pixels * cpad;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i % cpad);
    y[i] = fmaf(x[i], scale[c], shift[c]);
  }
}

// Depthwise convolution, NHWC, four channels per thread (16-B loads along C).
// w is [kh*kw][cpad]; bias [cpad]; residual NHWC like y.  Idx = int when the element count
// fits: the 64-bit divisions of the index decomposition would otherwise dominate.
template <typename Idx>
__global__ void depthwise_kernel(const float4* __restrict__ x, const float4* __restrict__ w,
                                 const float4* __restrict__ bias, const float4* __restrict__ res,
                                 float4* __restrict__ y, int n, int h, int wd, int c4, int oh, int ow, int kh, int kw,
                                 int sh, int sw, int ph, int pw, int dh, int dw, int act, int round_out) {
  const Idx total = (Idx)n * oh * ow * c4;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const int cq = (int)(i % c4);
    Idx t = i / c4;
    const int ox = (int)(t % ow);
    t /= ow;
    const int oy = (int)(t % oh);
    const int b = (int)(t / oh);
    float4 acc = make_float4(0, 0, 0, 0);
    for (int r = 0; r < kh; ++r) {
      const int iy = oy * sh - ph + r * dh;
      if (iy < 0 || iy >= h) continue;
      for (int s = 0; s < kw; ++s) {
        const int ix = ox * sw - pw + s * dw;
        if (ix < 0 || ix >= wd) continue;
        const float4 v = x[(((size_t)b * h + iy) * wd + ix) * c4 + cq];
        const float4 k = w[(size_t)(r * kw + s) * c4 + cq];
        acc.x = fmaf(v.x, k.x, acc.x);
        acc.y = fmaf(v.y, k.y, acc.y);
        acc.z = fmaf(v.z, k.z, acc.z);
        acc.w = fmaf(v.w, k.w, acc.w);
      }
    }
    if (bias) {
      const float4 bb = bias[cq];
      acc.x += bb.x;
      acc.y += bb.y;
      acc.z += bb.z;
      acc.w += bb.w;
    }
    if (res && (act == 4 || act == 5)) {
      const float4 rr = res[i];
      acc.x += rr.x;
      acc.y += rr.y;
      acc.z += rr.z;
      acc.w += rr.w;
    }
    acc.x = apply_act(acc.x, act);
    acc.y = apply_act(acc.y, act);
    acc.z = apply_act(acc.z, act);
    acc.w = apply_act(acc.w, act);
    if (round_out) {
      acc.x = to_tf32_rna(acc.x);
      acc.y = to_tf32_rna(acc.y);
      acc.z = to_tf32_rna(acc.z);
      acc.w = to_tf32_rna(acc.w);
    }
    y[i] = acc;
  }
}

// Depthwise 3x3 convolution (dilation 1, stride S = 1 or 2), NHWC, persistent CTAs.  A work
// unit is a tile of 8 x TW output pixels (TW = 16 at stride 1, 8 at stride 2) x 32 channels of
// one image.  One thread per CTA loads each unit's input window (its halo included) with a
// single 4-D TMA box -- each pixel's 32-channel slice is one 128-B line, out-of-range pixels
// and channels arrive as zeros, which is the convolution's zero padding -- into a ring of
// shared-memory buffers, up to three units ahead of the one being computed, so that HBM sees
// each input byte about once (the halo comes from L2) and enough bytes are in flight per SM to
// keep it streaming.  Thread (block, q) computes channel quad q of a block of RB x CB output
// pixels (2 x 2 at stride 1, 2 x 1 at stride 2), reading each window pixel of the block once
// from shared memory, with the taps accumulated in the order r, then s for every output; the
// epilogue is depthwise_kernel's (bias, residual, activation, tf32 rounding).  The 9 weights
// of a channel group stay in registers while the CTA's consecutive units share it.
// w is [9][cpad], bias [cpad], residual NHWC like y.  Waits are bounded; on expiry the CTA
// raises *err (code 4) and stops.
constexpr int kDwThreads = 256;
template <int S>
struct DwTile {
  static constexpr int TH = 8, TW = S == 1 ? 16 : 8;
  static constexpr int IH = (TH - 1) * S + 3, IW = (TW - 1) * S + 3;
  static constexpr uint32_t BYTES = IH * IW * 128;  // one window: IH x IW pixels x 32 channels
  static constexpr int RB = 2, CB = S == 1 ? 2 : 1;  // output block of one thread
  static constexpr int BX = TW / CB;                 // blocks per tile row
  static constexpr int BR = (RB - 1) * S + 3, BC = (CB - 1) * S + 3;  // window rows / columns a block reads
  static_assert((TH / RB) * BX * 8 == kDwThreads, "one block per thread");
  // Window buffers per CTA (loads run BUFS - 1 units ahead) and CTAs per SM: two CTAs of
  // 128 registers a thread (a 2 x 2 block keeps 16 window pixels, 4 accumulators and the 9
  // weights live); 4 x 23 KB or 3 x 37 KB of windows each.
  static constexpr int BUFS = S == 1 ? 4 : 3;
  static constexpr int MIN_CTAS = 2;
};

//
// POOL: the same tiles, windows and ring compute a 3x3 MaxPool instead (SPINN/run_time/ops/
// pool/maxpool.c:5-49): the maximum over the taps inside the image, starting from the
// reference's -1e30 (the TMA zero fill of padding positions is masked, not maxed).
template <int S, bool POOL = false>
__global__ void __launch_bounds__(kDwThreads, DwTile<S>::MIN_CTAS) depthwise3x3_tma_kernel(
    const __grid_constant__ CUtensorMap mx, const float4* __restrict__ w, const float4* __restrict__ bias,
    const float4* __restrict__ res, float4* __restrict__ y, int n, int c4, int oh, int ow, int ph, int pw,
    int tiles_x, int tiles_y, int groups, int act, int round_out, int* err, int h = 0, int wd = 0) {
  using T = DwTile<S>;
  extern __shared__ uint8_t dw_raw[];
  float4* buf = reinterpret_cast<float4*>((reinterpret_cast<uintptr_t>(dw_raw) + 127) & ~uintptr_t(127));
  __shared__ __align__(8) uint64_t full[T::BUFS];
  __shared__ volatile int abort_flag;
  // 32-bit unit arithmetic (the launcher keeps the unit count below 2^31): a 64-bit division
  // costs ~100 instructions, and every thread decodes its unit
  const int units = groups * n * tiles_y * tiles_x;
  // channel group fastest: CTAs working at the same time read every 128-B channel slice of
  // the same pixels, so DRAM sees whole pixel rows (c x 4 bytes) instead of one slice of each
  auto unit_coords = [&](int u, int* g, int* b, int* ty, int* tx) {
    *g = u % groups;
    int r = u / groups;
    *tx = r % tiles_x;
    r /= tiles_x;
    *ty = r % tiles_y;
    *b = r / tiles_y;
  };
  // thread 0's record of loads in flight: bit s set while buffer s awaits the phase in bit s of armed_ph
  uint32_t armed = 0, armed_ph = 0;
  auto issue = [&](int u, int it) {  // unit u is the CTA's it-th: buffer it % BUFS, phase (it / BUFS) & 1
    int g, b, ty, tx;
    unit_coords(u, &g, &b, &ty, &tx);
    const int slot = it % T::BUFS;
    mbar_arrive_expect_tx(&full[slot], T::BYTES);
    tma_load_4d(&mx, &full[slot], buf + (size_t)slot * (T::BYTES / 16), g * 32, tx * T::TW * S - pw,
                ty * T::TH * S - ph, b);
    armed |= 1u << slot;
    armed_ph = (armed_ph & ~(1u << slot)) | ((uint32_t)((it / T::BUFS) & 1) << slot);
  };
  if (threadIdx.x == 0) {
    for (int sl = 0; sl < T::BUFS; ++sl) mbar_init(&full[sl], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    prefetch_tmap(&mx);
    for (int k = 0; k < T::BUFS - 1; ++k)
      if ((long)blockIdx.x + (long)k * gridDim.x < units) issue((int)(blockIdx.x + k * gridDim.x), k);
  }
  const int q = threadIdx.x & 7, blk = threadIdx.x >> 3;
  const int by = blk / T::BX, bx = blk - by * T::BX;  // block origin: output row RB*by, column CB*bx of the tile
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  int wg = -1;  // channel quad whose weights are in registers
  float4 k[9];
  int it = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
    const int cur = it % T::BUFS;
    const long nu = (long)u + (long)(T::BUFS - 1) * gridDim.x;
    // the buffer of unit it + BUFS - 1 held unit it - 1, released by the last iteration's barrier
    if (threadIdx.x == 0 && nu < units) issue((int)nu, it + T::BUFS - 1);
    bool ok = mbar_wait(&full[cur], (uint32_t)((it / T::BUFS) & 1), &abort_flag, 4000000000ull);
    if (!__syncthreads_and(ok)) break;
    if (threadIdx.x == 0) armed &= ~(1u << cur);
    int g, b, ty, tx;
    unit_coords(u, &g, &b, &ty, &tx);
    const int qq = g * 8 + q;  // channel quad
    if (POOL && qq < c4) {
      const float4* win = buf + (size_t)cur * (T::BYTES / 16);
      const int iy0 = ty * T::TH * S - ph + by * T::RB * S, ix0 = tx * T::TW * S - pw + bx * T::CB * S;
      const float4 lo = make_float4(-1e30f, -1e30f, -1e30f, -1e30f);  // maxpool.c's initial value
      float4 acc[T::RB][T::CB];
#pragma unroll
      for (int i = 0; i < T::RB; ++i)
#pragma unroll
        for (int j = 0; j < T::CB; ++j) acc[i][j] = lo;
#pragma unroll
      for (int wr = 0; wr < T::BR; ++wr) {
        if ((unsigned)(iy0 + wr) >= (unsigned)h) continue;  // a padding row: no tap
#pragma unroll
        for (int wc = 0; wc < T::BC; ++wc) {
          if ((unsigned)(ix0 + wc) >= (unsigned)wd) continue;
          const float4 v = win[((by * T::RB * S + wr) * T::IW + bx * T::CB * S + wc) * 8 + q];
#pragma unroll
          for (int i = 0; i < T::RB; ++i) {
            const int r = wr - i * S;
            if (r < 0 || r > 2) continue;
#pragma unroll
            for (int j = 0; j < T::CB; ++j) {
              const int sc = wc - j * S;
              if (sc < 0 || sc > 2) continue;
              float4& m = acc[i][j];
              m.x = v.x > m.x ? v.x : m.x;
              m.y = v.y > m.y ? v.y : m.y;
              m.z = v.z > m.z ? v.z : m.z;
              m.w = v.w > m.w ? v.w : m.w;
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < T::RB; ++i)
#pragma unroll
        for (int j = 0; j < T::CB; ++j) {
          const int oy = ty * T::TH + by * T::RB + i, ox = tx * T::TW + bx * T::CB + j;
          if (oy < oh && ox < ow) y[(((size_t)b * oh + oy) * ow + ox) * c4 + qq] = acc[i][j];
        }
    } else if (!POOL && qq < c4) {
      if (qq != wg) {  // a new channel group: its weights
#pragma unroll
        for (int t = 0; t < 9; ++t) k[t] = __ldg(w + (size_t)t * c4 + qq);
        wg = qq;
      }
      const float4* win = buf + (size_t)cur * (T::BYTES / 16);
      const float4 bb = bias ? __ldg(bias + qq) : zero;
      float4 acc[T::RB][T::CB];
#pragma unroll
      for (int i = 0; i < T::RB; ++i)
#pragma unroll
        for (int j = 0; j < T::CB; ++j) acc[i][j] = zero;
      // window row wr of the block feeds output row i with tap r = wr - i*S (0..2); each of its
      // BC pixels feeds output column j with tap s = wc - j*S
#pragma unroll
      for (int wr = 0; wr < T::BR; ++wr) {
        float4 v[T::BC];
#pragma unroll
        for (int wc = 0; wc < T::BC; ++wc)
          v[wc] = win[((by * T::RB * S + wr) * T::IW + bx * T::CB * S + wc) * 8 + q];
#pragma unroll
        for (int i = 0; i < T::RB; ++i) {
          const int r = wr - i * S;
          if (r < 0 || r > 2) continue;
#pragma unroll
          for (int j = 0; j < T::CB; ++j)
#pragma unroll
            for (int s = 0; s < 3; ++s) {
              const float4 x = v[j * S + s], kk = k[r * 3 + s];
              acc[i][j].x = fmaf(x.x, kk.x, acc[i][j].x);
              acc[i][j].y = fmaf(x.y, kk.y, acc[i][j].y);
              acc[i][j].z = fmaf(x.z, kk.z, acc[i][j].z);
              acc[i][j].w = fmaf(x.w, kk.w, acc[i][j].w);
            }
        }
      }
#pragma unroll
      for (int i = 0; i < T::RB; ++i)
#pragma unroll
        for (int j = 0; j < T::CB; ++j) {
          const int oy = ty * T::TH + by * T::RB + i, ox = tx * T::TW + bx * T::CB + j;
          if (oy >= oh || ox >= ow) continue;
          float4 a = acc[i][j];
          if (bias) {
            a.x += bb.x;
            a.y += bb.y;
            a.z += bb.z;
            a.w += bb.w;
          }
          const size_t o = (((size_t)b * oh + oy) * ow + ox) * c4 + qq;
          if (res && (act == 4 || act == 5)) {
            const float4 rr = res[o];
            a.x += rr.x;
            a.y += rr.y;
            a.z += rr.z;
            a.w += rr.w;
          }
          a.x = apply_act(a.x, act);
          a.y = apply_act(a.y, act);
          a.z = apply_act(a.z, act);
          a.w = apply_act(a.w, act);
          if (round_out) {
            a.x = to_tf32_rna(a.x);
            a.y = to_tf32_rna(a.y);
            a.z = to_tf32_rna(a.z);
            a.w = to_tf32_rna(a.w);
          }
          y[o] = a;
        }
    }
    __syncthreads();  // every thread is done with buffer `cur`; it may be refilled
  }
  if (threadIdx.x == 0 && abort_flag) {
    // let every window still in flight land before the CTA's shared memory goes away
    volatile int dummy = 0;
    for (int sl = 0; sl < T::BUFS; ++sl)
      if (armed & (1u << sl)) mbar_wait(&full[sl], (armed_ph >> sl) & 1, &dummy, 200000000ull);
    atomicExch(err, 4);
  }
}

// Generic grouped direct convolution, NHWC, one output element per thread (CUDA cores).
// w is [oc][kh][kw][c/group].
__global__ void grouped_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               const float* __restrict__ bias, const float* __restrict__ res, float* __restrict__ y,
                               int n, int h, int wd, int c, int cpad, int oh, int ow, int oc, int ocpad, int kh, int kw,
                               int sh, int sw, int ph, int pw, int dh, int dw, int group, int act, int round_out) {
  const int cg = c / group, ocg = oc / group;
  const long total = (long)n * oh * ow * ocpad;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int o = (int)(i % ocpad);
    long t = i / ocpad;
    const int ox = (int)(t % ow);
    t /= ow;
    const int oy = (int)(t % oh);
    const int b = (int)(t / oh);
    if (o >= oc) {
      y[i] = 0.0f;
      continue;
    }
    const int g = o / ocg;
    float acc = 0.0f;
    for (int r = 0; r < kh; ++r) {
      const int iy = oy * sh - ph + r * dh;
      if (iy < 0 || iy >= h) continue;
      for (int s = 0; s < kw; ++s) {
        const int ix = ox * sw - pw + s * dw;
        if (ix < 0 || ix >= wd) continue;
        const float* xp = x + (((size_t)b * h + iy) * wd + ix) * cpad + g * cg;
        const float* wp = w + (((size_t)o * kh + r) * kw + s) * cg;
        for (int k = 0; k < cg; ++k) acc = fmaf(xp[k], wp[k], acc);
      }
    }
    if (bias) acc += bias[o];
    if (res && (act == 4 || act == 5)) acc += res[i];
    acc = apply_act(acc, act);
    y[i] = round_out ? to_tf32_rna(acc) : acc;
  }
}

template <typename Idx, bool W32>
__global__ void resize_nearest_kernel(const float4* __restrict__ x, float4* __restrict__ y, int n, int h, int w,
                                      int c4, int oh, int ow) {
  const Idx total = (Idx)n * oh * ow * c4;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const int cq = (int)(i % c4);
    Idx t = i / c4;
    const int ox = (int)(t % ow);
    t /= ow;
    const int oy = (int)(t % oh);
    const int b = (int)(t / oh);
    // 32-bit products when they fit (the launcher checks): a 64-bit division per element would
    // dominate this copy
    const int iy = W32 ? (int)((unsigned)oy * (unsigned)h / (unsigned)oh) : (int)((long)oy * h / oh);
    const int ix = W32 ? (int)((unsigned)ox * (unsigned)w / (unsigned)ow) : (int)((long)ox * w / ow);
    y[i] = x[(((size_t)b * h + iy) * w + ix) * c4 + cq];
  }
}

struct PermuteArgs {
  int ndim;
  long out_dims[8];
  long in_stride_of_out[8];  // input element stride for a step along each output dimension
};

__global__ void permute_kernel(const float* __restrict__ x, float* __restrict__ y, long total, PermuteArgs a) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    long rem = i, src = 0;
    for (int d = a.ndim - 1; d >= 0; --d) {
      const long c = rem % a.out_dims[d];
      rem /= a.out_dims[d];
      src += c * a.in_stride_of_out[d];
    }
    y[i] = x[src];
  }
}

// One warp per (outer, inner) row: max, sum of exp, normalise (three passes over dim).
__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ y, long outer, int dim, long inner) {
  const long rows = outer * inner;
  const int lane = threadIdx.x & 31;
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  for (long r = warp; r < rows; r += nwarps) {
    const long o = r / inner, in = r - o * inner;
    const float* xr = x + o * dim * inner + in;
    float* yr = y + o * dim * inner + in;
    float m = -INFINITY;
    for (int j = lane; j < dim; j += 32) m = fmaxf(m, xr[(long)j * inner]);
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sum = 0.0f;
    for (int j = lane; j < dim; j += 32) sum += expf(xr[(long)j * inner] - m);
    for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float inv = 1.0f / sum;
    for (int j = lane; j < dim; j += 32) yr[(long)j * inner] = expf(xr[(long)j * inner] - m) * inv;
  }
}

// Softmax over contiguous rows of dim <= 32 * NPL (inner == 1): each lane keeps its NPL values
// and their exponentials in registers, so the row is read once and expf runs once per element.
// Same operations in the same order as softmax_kernel (lane-strided sums, then the shuffle
// tree), so the results are identical.
template <int NPL>
__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y, long rows, int dim) {
  const int lane = threadIdx.x & 31;
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  for (long r = warp; r < rows; r += nwarps) {
    const float* xr = x + r * dim;
    float* yr = y + r * dim;
    float v[NPL];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      const int j = lane + 32 * k;
      v[k] = j < dim ? xr[j] : -INFINITY;
      m = fmaxf(m, v[k]);
    }
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      if (lane + 32 * k < dim) {
        v[k] = expf(v[k] - m);
        sum += v[k];
      }
    }
    for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      const int j = lane + 32 * k;
      if (j < dim) yr[j] = v[k] * inv;
    }
  }
}

__global__ void transpose_kernel(const float* __restrict__ x, float* __restrict__ y, int rows, int cols) {
  __shared__ float tile[32][33];
  const size_t off = (size_t)blockIdx.z * rows * cols;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, cc = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && cc < cols) ? x[off + (size_t)r * cols + cc] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int cc = c0 + i, r = r0 + threadIdx.x;
    if (cc < cols && r < rows) y[off + (size_t)cc * rows + r] = tile[threadIdx.x][i];
  }
}

template <typename Idx>
__global__ void split_tf32_kernel(const float* __restrict__ src, float* __restrict__ dst, Idx rows, int cols,
                                  int src_ld, int seg, int dst_ld, int o0, int o1, int o2) {
  const Idx total = rows * cols;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const Idx r = i / cols;  // Idx = int when the element count fits: no 64-bit division per element
    const int c = (int)(i - r * cols);
    const float v = src[(size_t)r * src_ld + c];
    const float hi = to_tf32_rna(v), lo = to_tf32_rna(v - hi);
    float* d = dst + (size_t)r * dst_ld + c;
    d[0] = o0 ? lo : hi;
    d[seg] = o1 ? lo : hi;
    d[2 * (long)seg] = o2 ? lo : hi;
  }
}

__global__ void round_tf32_kernel(float* x, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    x[i] = to_tf32_rna(x[i]);
}

}  // namespace

#define SPINN_LAUNCH_CHECK()                                                        \
  do {                                                                              \
    cudaError_t e_ = cudaGetLastError();                                            \
    if (e_ != cudaSuccess) {                                                        \
      set_error("%s: launch failed: %s", __func__, cudaGetErrorString(e_));         \
      return SPINN_CUDA_ECUDA;                                                      \
    }                                                                               \
    return 0;                                                                       \
  } while (0)

int launch_nchw_to_nhwc(const float* x, float* y, int n, int c, int h, int w, int cpad, cudaStream_t s,
                        int round_tf32) {
  const int hw = h * w;
  dim3 grid((hw + 31) / 32, (cpad + 31) / 32, n), block(32, 8);
  nchw_to_nhwc_kernel<<<grid, block, 0, s>>>(x, y, c, hw, cpad, round_tf32);
  SPINN_LAUNCH_CHECK();
}

int launch_space_to_depth2(const float* x, float* y, int n, int c, int h, int w, int h2, int w2, int ph, int pw,
                           cudaStream_t s, int round_tf32) {
  SPINN_CHECK_ARG(c >= 1 && c <= 4, "space_to_depth2: %d channels (at most 4)", c);
  const long work = (long)n * h2 * w2;
  const long span = (long)grid_for(work, kEltThreads) * kEltThreads;  // the loop index reaches work + span
  if (work < (1l << 31) - span)
    space_to_depth2_kernel<int><<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(
        x, reinterpret_cast<float4*>(y), n, c, h, w, h2, w2, ph, pw, round_tf32);
  else
    space_to_depth2_kernel<long><<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(
        x, reinterpret_cast<float4*>(y), n, c, h, w, h2, w2, ph, pw, round_tf32);
  SPINN_LAUNCH_CHECK();
}

int launch_nhwc_to_nchw(const float* x, float* y, int n, int c, int h, int w, int cpad, cudaStream_t s) {
  const int hw = h * w;
  dim3 grid((hw + 31) / 32, (c + 31) / 32, n), block(32, 8);
  nhwc_to_nchw_kernel<<<grid, block, 0, s>>>(x, y, c, hw, cpad);
  SPINN_LAUNCH_CHECK();
}

template <int S, bool POOL>
int launch_depthwise3x3_tma(const float* x, const float* w, const float* bias, const float* res, float* y, int n,
                            int h, int wd, int cpad, int oh, int ow, int ph, int pw, int act, int round_out, int dev,
                            cudaStream_t s);

int launch_maxpool_nhwc(const float* x, float* y, int n, int h, int w, int cpad, int oh, int ow, int kh, int kw,
                        int sh, int sw, int ph, int pw, cudaStream_t s) {
  SPINN_CHECK_ARG(cpad % 4 == 0, "maxpool: channel stride %d not a multiple of 4", cpad);
  // 3x3 stride 2 through the TMA window ring of the depthwise kernel (padding taps masked)
  if (kh == 3 && kw == 3 && sh == 2 && sw == 2 && ph >= 0 && pw >= 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    int dev = 0;
    SPINN_CUDA_TRY(cudaGetDevice(&dev));
    return launch_depthwise3x3_tma<2, true>(x, nullptr, nullptr, nullptr, y, n, h, w, cpad, oh, ow, ph, pw, 0, 0, dev, s);
  }
  // The tiled kernel needs every output window to hold at least one real tap (pads <= 1 with
  // the ONNX output size), which the -1e30 fill relies on like the generic kernel's skip.
  if (kh == 3 && kw == 3 && sh == 2 && sw == 2 && cpad / 4 <= kPoolMaxC4 && ph >= 0 && ph <= 1 && pw >= 0 &&
      pw <= 1 && (oh - 1) * 2 - ph < h && (ow - 1) * 2 - pw < w && n <= 65535) {
    dim3 grid((ow + kPoolTX - 1) / kPoolTX, (oh + kPoolTY - 1) / kPoolTY, n);
    maxpool3s2_tile_kernel<<<grid, kPoolThreads, 0, s>>>(reinterpret_cast<const float4*>(x),
                                                         reinterpret_cast<float4*>(y), h, w, cpad / 4, oh, ow, ph, pw);
    SPINN_LAUNCH_CHECK();
  }
  const long work = (long)n * oh * ow * (cpad / 4);
  if (work < (1l << 31) - (long)grid_for(work, kEltThreads) * kEltThreads)
    maxpool_nhwc_kernel<int><<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n, h, w, cpad / 4, oh, ow, kh, kw, sh, sw, ph,
        pw);
  else
    maxpool_nhwc_kernel<long><<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n, h, w, cpad / 4, oh, ow, kh, kw, sh, sw, ph,
        pw);
  SPINN_LAUNCH_CHECK();
}

int launch_wait_expiry_selftest(int* err, uint64_t timeout_ns, cudaStream_t s) {
  SPINN_CHECK_ARG(err != nullptr && timeout_ns > 0 && timeout_ns <= 1000000000ull,
                  "wait self-test: timeout %llu ns outside (0, 1 s]", (unsigned long long)timeout_ns);
  wait_expiry_kernel<<<1, 32, 0, s>>>(err, (unsigned long long)timeout_ns);
  SPINN_LAUNCH_CHECK();
}

int launch_topk(const float* x, long rows, int n, int k, float* vals, int64_t* idx, cudaStream_t s) {
  SPINN_CHECK_ARG(n >= 1 && n <= kTopkMaxN, "topk: row length %d outside [1, %d]", n, kTopkMaxN);
  SPINN_CHECK_ARG(k >= 0 && k <= n, "topk: k=%d outside [0, %d]", k, n);
  SPINN_CHECK_ARG(rows >= 0 && rows <= 0x7FFFFFFF, "topk: %ld rows", rows);
  if (rows == 0 || k == 0) return 0;
  int npow2 = 1;
  while (npow2 < n) npow2 <<= 1;
  const size_t smem = (size_t)npow2 * 8;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  SPINN_CUDA_TRY(cudaGetDevice(&dev));
  if (!(configured.load() & (1ull << (dev & 63)))) {
    SPINN_CUDA_TRY(cudaFuncSetAttribute(topk_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)((size_t)kTopkMaxN * 8)));
    configured.fetch_or(1ull << (dev & 63));
  }
  topk_rows_kernel<<<(unsigned)rows, 1024, smem, s>>>(x, n, k, npow2, vals, idx);
  SPINN_LAUNCH_CHECK();
}

int launch_copy_rows(const float* src, int src_ld, float* dst, int dst_ld, long rows, int width, int fill_to,
                     cudaStream_t s) {
  SPINN_CHECK_ARG(width >= 0 && fill_to >= width && src_ld >= width && dst_ld >= fill_to && rows >= 0,
                  "copy_rows: width %d fill %d src_ld %d dst_ld %d", width, fill_to, src_ld, dst_ld);
  if (rows == 0 || fill_to == 0) return 0;
  const bool v4 = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0 &&
                  src_ld % 4 == 0 && dst_ld % 4 == 0 && width % 4 == 0 && fill_to % 4 == 0;
  const long work = rows * (v4 ? fill_to / 4 : fill_to);
  const int grid = grid_for(work, kEltThreads);
  const bool small = work < (1l << 31) - (long)grid * kEltThreads;
  if (v4 && small)
    copy_rows_kernel<4, int><<<grid, kEltThreads, 0, s>>>(src, src_ld, dst, dst_ld, (int)rows, width, fill_to);
  else if (v4)
    copy_rows_kernel<4, long><<<grid, kEltThreads, 0, s>>>(src, src_ld, dst, dst_ld, rows, width, fill_to);
  else if (small)
    copy_rows_kernel<1, int><<<grid, kEltThreads, 0, s>>>(src, src_ld, dst, dst_ld, (int)rows, width, fill_to);
  else
    copy_rows_kernel<1, long><<<grid, kEltThreads, 0, s>>>(src, src_ld, dst, dst_ld, rows, width, fill_to);
  SPINN_LAUNCH_CHECK();
}

int launch_concat_rows(const CatParts& parts, float* dst, int dst_ld, long rows, int fill_to, cudaStream_t s) {
  SPINN_CHECK_ARG(parts.n >= 1 && parts.n <= kCatMaxParts && fill_to % 4 == 0 && dst_ld >= fill_to && dst_ld % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
                  "concat_rows: %d parts, fill %d, ld %d", parts.n, fill_to, dst_ld);
  for (int k = 0; k < parts.n; ++k)
    SPINN_CHECK_ARG(parts.off[k] % 4 == 0 && parts.width[k] % 4 == 0 && parts.ld[k] % 4 == 0 &&
                        parts.ld[k] >= parts.width[k] && parts.off[k] + parts.width[k] <= fill_to &&
                        (reinterpret_cast<uintptr_t>(parts.src[k]) & 15) == 0,
                    "concat_rows: part %d misaligned", k);
  if (rows == 0 || fill_to == 0) return 0;
  const long work = rows * (fill_to / 4);
  const int grid = grid_for(work, kEltThreads);
  if (work < (1l << 31) - (long)grid * kEltThreads)
    concat_rows_kernel<int><<<grid, kEltThreads, 0, s>>>(parts, dst, dst_ld, (int)rows, fill_to);
  else
    concat_rows_kernel<long><<<grid, kEltThreads, 0, s>>>(parts, dst, dst_ld, rows, fill_to);
  SPINN_LAUNCH_CHECK();
}

int launch_split_rows(const SplitParts& parts, const float* src, int src_ld, long rows, cudaStream_t s) {
  SPINN_CHECK_ARG(parts.n >= 1 && parts.n <= kCatMaxParts && src_ld % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0,
                  "split_rows: %d parts, ld %d", parts.n, src_ld);
  int width = 0;
  for (int k = 0; k < parts.n; ++k) {
    SPINN_CHECK_ARG(parts.off[k] == width && parts.width[k] % 4 == 0 && parts.ld[k] == parts.width[k] &&
                        (reinterpret_cast<uintptr_t>(parts.dst[k]) & 15) == 0,
                    "split_rows: part %d not dense and float4-aligned", k);
    width += parts.width[k];
  }
  SPINN_CHECK_ARG(width <= src_ld, "split_rows: parts wider than the source row");
  if (rows == 0 || width == 0) return 0;
  const long work = rows * (width / 4);
  const int grid = grid_for(work, kEltThreads);
  if (work < (1l << 31) - (long)grid * kEltThreads)
    split_rows_kernel<int><<<grid, kEltThreads, 0, s>>>(parts, src, src_ld, (int)rows, width);
  else
    split_rows_kernel<long><<<grid, kEltThreads, 0, s>>>(parts, src, src_ld, rows, width);
  SPINN_LAUNCH_CHECK();
}

int launch_gather_rows(const GatherPieces& g, float* dst, int n, int ctot, int ltot, cudaStream_t s) {
  SPINN_CHECK_ARG(g.n >= 1 && g.n <= kGatherMaxPieces && n >= 0 && ctot >= 0 && ltot >= 0,
                  "gather_rows: %d pieces", g.n);
  GatherTiles t{};
  t.tile0[0] = 0;
  for (int k = 0; k < g.n; ++k) {
    SPINN_CHECK_ARG(g.chans[k] >= 0 && g.len[k] >= 0 && g.dst_c[k] >= 0 && g.dst_c[k] + g.chans[k] <= ctot &&
                        g.dst_l[k] >= 0 && g.dst_l[k] + g.len[k] <= ltot && g.c0[k] >= 0 &&
                        (g.nhwc[k] ? g.c0[k] + g.chans[k] <= g.ld[k] : g.len[k] <= g.ld[k]),
                    "gather_rows: piece %d out of range", k);
    t.ctiles[k] = (g.chans[k] + 31) / 32;
    t.ltiles[k] = (g.len[k] + kGatherTL - 1) / kGatherTL;
    SPINN_CHECK_ARG((long)n * t.ctiles[k] * t.ltiles[k] < (1l << 31) &&
                        (long)(g.nhwc[k] ? g.len[k] : g.chans[k]) * g.ld[k] < (1l << 31) && 32l * ltot < (1l << 31),
                    "gather_rows: piece %d too large for 32-bit offsets", k);
    t.tile0[k + 1] = t.tile0[k] + (long)n * t.ctiles[k] * t.ltiles[k];
  }
  const long total = t.tile0[g.n];
  if (total == 0) return 0;
  const int grid = (int)std::min<long>(total, 148L * 8);
  gather_rows_kernel<<<grid, dim3(32, 8), 0, s>>>(g, t, dst, n, ctot, ltot);
  SPINN_LAUNCH_CHECK();
}

int launch_avgpool_nhwc(const float* x, float* y, int n, int h, int w, int cpad, int oh, int ow, int kh, int kw,
                        int sh, int sw, int ph, int pw, int count_include_pad, cudaStream_t s) {
  SPINN_CHECK_ARG(cpad % 4 == 0, "avgpool: channel stride %d not a multiple of 4", cpad);
  const long work = (long)n * oh * ow * (cpad / 4);
  avgpool_nhwc_kernel<<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(
      reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n, h, w, cpad / 4, oh, ow, kh, kw, sh, sw, ph, pw,
      count_include_pad);
  SPINN_LAUNCH_CHECK();
}

int launch_gap_nhwc(const float* x, float* y, int n, int hw, int cpad, cudaStream_t s, int round_tf32) {
  const long work = (long)n * cpad;
  gap_nhwc_kernel<<<grid_for(work, 128), 128, 0, s>>>(x, y, n, hw, cpad, round_tf32);
  SPINN_LAUNCH_CHECK();
}

int launch_binary(const float* a, long na, const float* b, long nb, float* y, long n, int op, int act, cudaStream_t s) {
  SPINN_CHECK_ARG(na > 0 && nb > 0, "binary: empty operand");
  if (na == n && nb == n && n % 4 == 0 &&
      ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(y)) & 15) == 0) {
    binary4_kernel<<<grid_for(n / 4, kEltThreads), kEltThreads, 0, s>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(y), n / 4, op,
        act);
    SPINN_LAUNCH_CHECK();
  }
  binary_kernel<<<grid_for(n, kEltThreads), kEltThreads, 0, s>>>(a, na, b, nb, y, n, op, act);
  SPINN_LAUNCH_CHECK();
}

int launch_unary(const float* x, float* y, long n, int op, cudaStream_t s) {
  unary_kernel<<<grid_for(n, kEltThreads), kEltThreads, 0, s>>>(x, y, n, op);
  SPINN_LAUNCH_CHECK();
}

int launch_channel_affine_nhwc(const float* x, float* y, long pixels, int cpad, const float* scale,
                               const float* shift, cudaStream_t s) {
  channel_affine_kernel<<<grid_for(pixels * cpad, kEltThreads), kEltThreads, 0, s>>>(x, y, pixels, cpad, scale, shift);
  SPINN_LAUNCH_CHECK();
}

template <int S, bool POOL = false>
int launch_depthwise3x3_tma(const float* x, const float* w, const float* bias, const float* res, float* y, int n,
                            int h, int wd, int cpad, int oh, int ow, int ph, int pw, int act, int round_out, int dev,
                            cudaStream_t s) {
  using T = DwTile<S>;
  CUtensorMap mx;
  int rc = encode_nhwc_window(&mx, x, n, h, wd, cpad, 32, T::IW, T::IH);
  if (rc) return rc;
  const int tiles_x = (ow + T::TW - 1) / T::TW, tiles_y = (oh + T::TH - 1) / T::TH;
  const int groups = (cpad / 4 + 7) / 8;
  const long units = (long)groups * n * tiles_y * tiles_x;
  SPINN_CHECK_ARG(units < (1l << 31) - 2l * 148 * 8 * T::BUFS, "depthwise: %ld work units", units);
  const int smem = (int)(T::BUFS * T::BYTES + 128);
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    SPINN_CUDA_TRY(
        cudaFuncSetAttribute(depthwise3x3_tma_kernel<S, POOL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured.fetch_or(bit);
  }
  int per_sm = 0;
  SPINN_CUDA_TRY(
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, depthwise3x3_tma_kernel<S, POOL>, kDwThreads, smem));
  const long grid = std::min<long>(units, (long)sm_count(dev) * std::max(per_sm, 1));
  if (grid <= 0) return 0;
  depthwise3x3_tma_kernel<S, POOL><<<(int)grid, kDwThreads, smem, s>>>(
      mx, reinterpret_cast<const float4*>(w), reinterpret_cast<const float4*>(bias),
      reinterpret_cast<const float4*>(res), reinterpret_cast<float4*>(y), n, cpad / 4, oh, ow, ph, pw, tiles_x,
      tiles_y, groups, act, round_out, device_error_flag(dev), h, wd);
  SPINN_LAUNCH_CHECK();
}

int launch_depthwise_nhwc(const float* x, const float* w, const float* bias, const float* res, float* y, int n, int h,
                          int wd, int cpad, int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw, int dh,
                          int dw, int act, int round_out, cudaStream_t s) {
  SPINN_CHECK_ARG(cpad % 4 == 0, "depthwise: channel stride %d not a multiple of 4", cpad);
  if (kh == 3 && kw == 3 && dh == 1 && dw == 1 && sh == sw && (sh == 1 || sh == 2) && ph >= 0 && pw >= 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    int dev = 0;
    SPINN_CUDA_TRY(cudaGetDevice(&dev));
    return sh == 1 ? launch_depthwise3x3_tma<1>(x, w, bias, res, y, n, h, wd, cpad, oh, ow, ph, pw, act, round_out,
                                                 dev, s)
                   : launch_depthwise3x3_tma<2>(x, w, bias, res, y, n, h, wd, cpad, oh, ow, ph, pw, act, round_out,
                                                 dev, s);
  }
  const long work = (long)n * oh * ow * (cpad / 4);
  const long span = (long)grid_for(work, kEltThreads) * kEltThreads;  // the loop index reaches work + span
  if (work < (1l << 31) - span)
    depthwise_kernel<int><<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(w), reinterpret_cast<const float4*>(bias),
        reinterpret_cast<const float4*>(res), reinterpret_cast<float4*>(y), n, h, wd, cpad / 4, oh, ow, kh, kw, sh, sw,
        ph, pw, dh, dw, act, round_out);
  else
    depthwise_kernel<long><<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(w), reinterpret_cast<const float4*>(bias),
        reinterpret_cast<const float4*>(res), reinterpret_cast<float4*>(y), n, h, wd, cpad / 4, oh, ow, kh, kw, sh, sw,
        ph, pw, dh, dw, act, round_out);
  SPINN_LAUNCH_CHECK();
}

int launch_grouped_nhwc(const float* x, const float* w, const float* bias, const float* res, float* y, int n, int h,
                        int wd, int c, int cpad, int oh, int ow, int oc, int ocpad, int kh, int kw, int sh, int sw,
                        int ph, int pw, int dh, int dw, int group, int act, int round_out, cudaStream_t s) {
  SPINN_CHECK_ARG(group >= 1 && c % group == 0 && oc % group == 0, "grouped conv: bad group %d", group);
  const long work = (long)n * oh * ow * ocpad;
  grouped_kernel<<<grid_for(work, kEltThreads), kEltThreads, 0, s>>>(x, w, bias, res, y, n, h, wd, c, cpad, oh, ow, oc,
                                                                    ocpad, kh, kw, sh, sw, ph, pw, dh, dw, group, act,
                                                                    round_out);
  SPINN_LAUNCH_CHECK();
}

int launch_resize_nearest_nhwc(const float* x, float* y, int n, int h, int w, int cpad, int oh, int ow,
                               cudaStream_t s) {
  SPINN_CHECK_ARG(cpad % 4 == 0, "resize: channel stride %d not a multiple of 4", cpad);
  const long work = (long)n * oh * ow * (cpad / 4);
  const long span = (long)grid_for(work, kEltThreads) * kEltThreads;  // the loop index reaches work + span
  const bool w32 = (long)oh * h < (1l << 32) && (long)ow * w < (1l << 32);
  const float4* xv = reinterpret_cast<const float4*>(x);
  float4* yv = reinterpret_cast<float4*>(y);
  const int g = grid_for(work, kEltThreads), c4 = cpad / 4;
  if (work < (1l << 31) - span) {
    if (w32)
      resize_nearest_kernel<int, true><<<g, kEltThreads, 0, s>>>(xv, yv, n, h, w, c4, oh, ow);
    else
      resize_nearest_kernel<int, false><<<g, kEltThreads, 0, s>>>(xv, yv, n, h, w, c4, oh, ow);
  } else {
    if (w32)
      resize_nearest_kernel<long, true><<<g, kEltThreads, 0, s>>>(xv, yv, n, h, w, c4, oh, ow);
    else
      resize_nearest_kernel<long, false><<<g, kEltThreads, 0, s>>>(xv, yv, n, h, w, c4, oh, ow);
  }
  SPINN_LAUNCH_CHECK();
}

int launch_permute(const float* x, float* y, int ndim, const uint32_t* dims, const uint8_t* perm, cudaStream_t s) {
  SPINN_CHECK_ARG(ndim >= 1 && ndim <= 8, "transpose: %d dimensions", ndim);
  PermuteArgs a;
  a.ndim = ndim;
  long in_stride[8];
  in_stride[ndim - 1] = 1;
  for (int d = ndim - 2; d >= 0; --d) in_stride[d] = in_stride[d + 1] * dims[d + 1];
  long total = 1;
  for (int d = 0; d < ndim; ++d) {
    SPINN_CHECK_ARG(perm[d] < ndim, "transpose: bad permutation");
    a.out_dims[d] = dims[perm[d]];
    a.in_stride_of_out[d] = in_stride[perm[d]];
    total *= a.out_dims[d];
  }
  permute_kernel<<<grid_for(total, kEltThreads), kEltThreads, 0, s>>>(x, y, total, a);
  SPINN_LAUNCH_CHECK();
}

int launch_softmax(const float* x, float* y, long outer, int dim, long inner, cudaStream_t s) {
  const long rows = outer * inner;
  if (inner == 1 && dim <= 32 * 16) {
    softmax_rows_kernel<16><<<grid_for(rows * 32, kEltThreads), kEltThreads, 0, s>>>(x, y, rows, dim);
    SPINN_LAUNCH_CHECK();
  }
  softmax_kernel<<<grid_for(rows * 32, kEltThreads), kEltThreads, 0, s>>>(x, y, outer, dim, inner);
  SPINN_LAUNCH_CHECK();
}

int launch_transpose(const float* x, float* y, int batch, int rows, int cols, cudaStream_t s) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32, batch), block(32, 8);
  transpose_kernel<<<grid, block, 0, s>>>(x, y, rows, cols);
  SPINN_LAUNCH_CHECK();
}

int launch_split_tf32(const float* src, float* dst, long rows, int cols, int src_ld, int seg, int dst_ld, int o0,
                      int o1, int o2, cudaStream_t s) {
  SPINN_CHECK_ARG(seg >= cols && src_ld >= cols && dst_ld >= 3 * seg, "split_tf32: bad strides");
  const long work = rows * cols;
  const int g = grid_for(work, kEltThreads);
  if (work < (1l << 31) - (long)g * kEltThreads)
    split_tf32_kernel<int><<<g, kEltThreads, 0, s>>>(src, dst, (int)rows, cols, src_ld, seg, dst_ld, o0, o1, o2);
  else
    split_tf32_kernel<long><<<g, kEltThreads, 0, s>>>(src, dst, rows, cols, src_ld, seg, dst_ld, o0, o1, o2);
  SPINN_LAUNCH_CHECK();
}

int launch_round_tf32(float* x, long n, cudaStream_t s) {
  round_tf32_kernel<<<grid_for(n, kEltThreads), kEltThreads, 0, s>>>(x, n);
  SPINN_LAUNCH_CHECK();
}

}  // namespace spinn
