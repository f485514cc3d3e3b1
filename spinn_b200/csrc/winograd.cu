// winograd.cu -- 3x3 stride-1 convolution by Winograd F(4x4,3x3) on NHWC tensors.
//
//   V[xi][t][c]  = (B^T d_t,c B)[xi]        input transform, one 6x6 patch per 4x4 output tile
//   M[xi]        = V[xi] * U[xi]^T          36 tcgen05 GEMMs (tiled mode), U = G g G^T, each a
//                                           split-tf32 product (see winograd_f43_weights)
//   y[tile]      = A^T M[.][t][o] A + bias (+ residual) -> activation -> (tf32 rounding)
//
// The reference's Winograd is F(2x2,3x3) (SPINN/run_time/ops/conv/winograd.c:16-210) and is
// disabled in op_conv2d (conv2d.c:155); F(4x4,3x3) uses Lavin & Gray's interpolation points
// {0, 1, -1, 2, -2, inf}:
//   B^T = [4 0 -5 0 1 0; 0 -4 -4 1 1 0; 0 4 -4 -1 1 0; 0 -2 -1 2 1 0; 0 2 -1 -2 1 0; 0 4 0 -5 0 1]
//   G   = [1/4 0 0; -1/6 -1/6 -1/6; -1/6 1/6 -1/6; 1/24 1/12 1/6; 1/24 -1/12 1/6; 0 0 1]
//   A^T = [1 1 1 1 1 0; 0 1 -1 2 -2 0; 0 1 1 4 4 0; 0 1 -1 8 -8 1]
// Transforms are HBM-bound: V and M are 36/16 of the input / output each, written and read
// once, so on B200 this path beats the implicit GEMM only where the convolution itself is
// far from the memory roofline; the planner uses it when asked (plan flag WINOGRAD).  Measured
// on B200 for the ResNet 3x3 shapes at batch 256 it is 1.5-3.7x slower than the implicit GEMM.
#include "internal.h"
#include "ptx.cuh"

namespace spinn {
namespace {

constexpr int kThreads = 256;

inline int grid_for(long work) {
  long b = (work + kThreads - 1) / kThreads;
  if (b < 1) b = 1;
  if (b > 148 * 32) b = 148 * 32;
  return (int)b;
}

// B^T d B on one 6x6 patch of one channel.
__device__ __forceinline__ void bt_d_b(const float d[6][6], float v[6][6]) {
  float t[6][6];
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    t[0][j] = 4.f * d[0][j] - 5.f * d[2][j] + d[4][j];
    t[1][j] = -4.f * d[1][j] - 4.f * d[2][j] + d[3][j] + d[4][j];
    t[2][j] = 4.f * d[1][j] - 4.f * d[2][j] - d[3][j] + d[4][j];
    t[3][j] = -2.f * d[1][j] - d[2][j] + 2.f * d[3][j] + d[4][j];
    t[4][j] = 2.f * d[1][j] - d[2][j] - 2.f * d[3][j] + d[4][j];
    t[5][j] = 4.f * d[1][j] - 5.f * d[3][j] + d[5][j];
  }
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    v[i][0] = 4.f * t[i][0] - 5.f * t[i][2] + t[i][4];
    v[i][1] = -4.f * t[i][1] - 4.f * t[i][2] + t[i][3] + t[i][4];
    v[i][2] = 4.f * t[i][1] - 4.f * t[i][2] - t[i][3] + t[i][4];
    v[i][3] = -2.f * t[i][1] - t[i][2] + 2.f * t[i][3] + t[i][4];
    v[i][4] = 2.f * t[i][1] - t[i][2] - 2.f * t[i][3] + t[i][4];
    v[i][5] = 4.f * t[i][1] - 5.f * t[i][3] + t[i][5];
  }
}

// A^T m A: 6x6 -> 4x4.
__device__ __forceinline__ void at_m_a(const float m[6][6], float y[4][4]) {
  float t[4][6];
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    t[0][j] = m[0][j] + m[1][j] + m[2][j] + m[3][j] + m[4][j];
    t[1][j] = m[1][j] - m[2][j] + 2.f * m[3][j] - 2.f * m[4][j];
    t[2][j] = m[1][j] + m[2][j] + 4.f * m[3][j] + 4.f * m[4][j];
    t[3][j] = m[1][j] - m[2][j] + 8.f * m[3][j] - 8.f * m[4][j] + m[5][j];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    y[i][0] = t[i][0] + t[i][1] + t[i][2] + t[i][3] + t[i][4];
    y[i][1] = t[i][1] - t[i][2] + 2.f * t[i][3] - 2.f * t[i][4];
    y[i][2] = t[i][1] + t[i][2] + 4.f * t[i][3] + 4.f * t[i][4];
    y[i][3] = t[i][1] - t[i][2] + 8.f * t[i][3] - 8.f * t[i][4] + t[i][5];
  }
}

// x NHWC [n][h][w][cpad] -> v [36][tiles][3*cpad]; one thread per (tile, channel).
__global__ void wino_input_kernel(const float* __restrict__ x, float* __restrict__ v, int n, int h, int w, int cpad,
                                  int th, int tw, int ph, int pw) {
  const long tiles = (long)n * th * tw;
  const long total = tiles * cpad;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i % cpad);
    const long t = i / cpad;
    const int tj = (int)(t % tw);
    const long r = t / tw;
    const int ti = (int)(r % th);
    const int b = (int)(r / th);
    const int y0 = ti * 4 - ph, x0 = tj * 4 - pw;
    float d[6][6], o[6][6];
#pragma unroll
    for (int a = 0; a < 6; ++a)
#pragma unroll
      for (int e = 0; e < 6; ++e) {
        const int yy = y0 + a, xx = x0 + e;
        d[a][e] = (yy >= 0 && yy < h && xx >= 0 && xx < w) ? x[(((size_t)b * h + yy) * w + xx) * cpad + c] : 0.0f;
      }
    bt_d_b(d, o);
    // split tf32: row of V' = [hi | lo | hi] over 3*cpad columns (see winograd_f43_weights)
#pragma unroll
    for (int a = 0; a < 6; ++a)
#pragma unroll
      for (int e = 0; e < 6; ++e) {
        const float hi = to_tf32_rna(o[a][e]);
        const float lo = to_tf32_rna(o[a][e] - hi);
        float* row = v + ((size_t)(a * 6 + e) * tiles + t) * (3 * (size_t)cpad);
        row[c] = hi;
        row[cpad + c] = lo;
        row[2 * cpad + c] = hi;
      }
  }
}

// m [36][tiles][ocpad] -> y NHWC [n][oh][ow][ocpad] with the sgemm_nn epilogue.
__global__ void wino_output_kernel(const float* __restrict__ m, const float* __restrict__ bias,
                                   const float* __restrict__ res, float* __restrict__ y, int n, int oh, int ow,
                                   int ocpad, int th, int tw, int act, int round_out) {
  const long tiles = (long)n * th * tw;
  const long total = tiles * ocpad;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int o = (int)(i % ocpad);
    const long t = i / ocpad;
    const int tj = (int)(t % tw);
    const long r = t / tw;
    const int ti = (int)(r % th);
    const int b = (int)(r / th);
    float mm[6][6], out[4][4];
#pragma unroll
    for (int a = 0; a < 6; ++a)
#pragma unroll
      for (int e = 0; e < 6; ++e) mm[a][e] = m[((size_t)(a * 6 + e) * tiles + t) * ocpad + o];
    at_m_a(mm, out);
    const float bv = bias ? bias[o] : 0.0f;
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int yy = ti * 4 + a, xx = tj * 4 + e;
        if (yy >= oh || xx >= ow) continue;
        const size_t idx = (((size_t)b * oh + yy) * ow + xx) * ocpad + o;
        float v = out[a][e] + bv;
        if (res && (act == 4 || act == 5)) v += res[idx];
        if (act == 1 || act == 5)
          v = v < 0.0f ? 0.0f : v;
        else if (act == 3)
          v = silu_fast(v);
        y[idx] = round_out ? to_tf32_rna(v) : v;
      }
  }
}

}  // namespace

void winograd_f43_weights(const float* w, int oc, int c, int cpad, int ocpad, int kpad, float* u) {
  // U[xi][o] = (G g G^T)[xi] as three K segments [U_hi | U_hi | U_lo] of cpad columns, so that
  // with V' = [V_hi | V_lo | V_hi] one GEMM gives V_hi U_hi + V_lo U_hi + V_hi U_lo: the
  // split-tf32 product, accurate to about fp32 (single tf32 operands lose ~3e-3 relative L2
  // through the transforms).  Stored [36][ocpad][kpad], kpad >= 3*cpad, zero padding.
  static const double G[6][3] = {{0.25, 0, 0},
                                 {-1.0 / 6, -1.0 / 6, -1.0 / 6},
                                 {-1.0 / 6, 1.0 / 6, -1.0 / 6},
                                 {1.0 / 24, 1.0 / 12, 1.0 / 6},
                                 {1.0 / 24, -1.0 / 12, 1.0 / 6},
                                 {0, 0, 1}};
  std::memset(u, 0, sizeof(float) * 36 * (size_t)ocpad * kpad);
  for (int o = 0; o < oc; ++o)
    for (int ch = 0; ch < c; ++ch) {
      const float* g = w + ((size_t)o * c + ch) * 9;
      double t[6][3];
      for (int i = 0; i < 6; ++i)
        for (int j = 0; j < 3; ++j) t[i][j] = G[i][0] * g[j] + G[i][1] * g[3 + j] + G[i][2] * g[6 + j];
      for (int i = 0; i < 6; ++i)
        for (int j = 0; j < 6; ++j) {
          const double v = t[i][0] * G[j][0] + t[i][1] * G[j][1] + t[i][2] * G[j][2];
          const float hi = host_round_tf32((float)v);
          const float lo = host_round_tf32((float)(v - (double)hi));
          float* row = u + ((size_t)(i * 6 + j) * ocpad + o) * kpad;
          row[ch] = hi;
          row[cpad + ch] = hi;
          row[2 * cpad + ch] = lo;
        }
    }
}

int winograd_f43_run(const WinogradArgs& a, cudaStream_t s) {
  SPINN_CHECK_ARG(a.cpad % 4 == 0 && a.ocpad % 4 == 0, "winograd: channel strides must be multiples of 4");
  const int th = (a.oh + 3) / 4, tw = (a.ow + 3) / 4;
  const long tiles = (long)a.n * th * tw;
  SPINN_CHECK_ARG(tiles <= 0x7FFFFFFF, "winograd: too many tiles");
  wino_input_kernel<<<grid_for(tiles * a.cpad), kThreads, 0, s>>>(a.x, a.v, a.n, a.h, a.w, a.cpad, th, tw, a.ph, a.pw);
  SPINN_CUDA_TRY(cudaGetLastError());
  for (int xi = 0; xi < 36; ++xi) {
    TcGemmArgs g;
    g.a_mode = 1;
    g.x = a.v + (size_t)xi * tiles * 3 * a.cpad;
    g.M = (int)tiles;
    g.K = 3 * a.cpad;
    g.lda = 3 * a.cpad;
    g.wt = a.u + (size_t)xi * a.ocpad * a.kpad;
    g.kpad = a.kpad;
    g.N = a.ocpad;
    g.y = a.m + (size_t)xi * tiles * a.ocpad;
    g.ldy = a.ocpad;
    int rc = tc_gemm_launch(g, s);
    if (rc) return rc;
  }
  wino_output_kernel<<<grid_for(tiles * a.ocpad), kThreads, 0, s>>>(a.m, a.bias, a.res, a.y, a.n, a.oh, a.ow, a.ocpad,
                                                                    th, tw, a.act, a.round_out);
  SPINN_CUDA_TRY(cudaGetLastError());
  return 0;
}

}  // namespace spinn
