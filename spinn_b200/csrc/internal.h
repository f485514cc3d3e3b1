// internal.h -- declarations shared by the translation units of libspinn_cuda.so.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/spinn_cuda.h"

namespace spinn {

// ------------------------------------------------------------------ errors
// Thread-local message of the last failure (spinn_cuda_last_error).
void set_error(const char* fmt, ...);
const char* get_error();

#define SPINN_CUDA_TRY(expr)                                                                \
  do {                                                                                      \
    cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess) {                                                                \
      ::spinn::set_error("%s:%d: %s: %s", __FILE__, __LINE__, #expr, cudaGetErrorString(e_)); \
      return SPINN_CUDA_ECUDA;                                                              \
    }                                                                                       \
  } while (0)

#define SPINN_CHECK_ARG(cond, ...)        \
  do {                                    \
    if (!(cond)) {                        \
      ::spinn::set_error(__VA_ARGS__);    \
      return SPINN_CUDA_EINVAL;           \
    }                                     \
  } while (0)

// ------------------------------------------------------------------ tensor maps
// Wrappers over cuTensorMapEncodeTiled / cuTensorMapEncodeIm2col obtained through
// cudaGetDriverEntryPoint (no link-time dependency on libcuda).  fp32 only.
int encode_tiled_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle);
// 3-D tiled map of `planes` row-major [outer][inner] matrices stored back to back.
int encode_tiled_3d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t planes,
                    uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);
// 4-D tiled map of an NHWC tensor [n][h][w][cpad] whose boxes are windows of box_h x box_w
// pixels x box_c channels (no swizzle; out-of-range pixels and channels read as zeros).
int encode_nhwc_window(CUtensorMap* map, const void* base, int n, int h, int w, int cpad, uint32_t box_c,
                       uint32_t box_w, uint32_t box_h);
int encode_im2col_4d(CUtensorMap* map, const void* base, int n, int h, int w, int c,
                     int lower_w, int lower_h, int upper_w, int upper_h, int channels_per_pixel,
                     int pixels_per_column, int stride_w, int stride_h, CUtensorMapSwizzle swizzle);

// Device properties cached per device.
int sm_count(int device);

// Device word that kernels set when a bounded wait expires (one per device).
int* device_error_flag(int device);
// Reads and clears the flag; SPINN_CUDA_ETIMEOUT if it was set.
int check_device_error_flag(int device, cudaStream_t stream);
// One-thread kernel whose mbarrier wait expires after timeout_ns (<= 1 s) and raises *err.
int launch_wait_expiry_selftest(int* err, uint64_t timeout_ns, cudaStream_t s);

// ------------------------------------------------------------------ tcgen05 GEMM / conv
// Y[M][ldy] = epilogue( A * W^T ), W stored K-major [N][kpad].
//   a_mode 0 (im2col): A is the implicit im2col matrix of an NHWC activation
//     x[n][h][w][cpad] for a (kh,kw) filter with stride/pad/dilation; M = n*oh*ow and
//     K index = ((r*kw)+s)*cpad + c.
//   a_mode 1 (tiled): A is a row-major [M][lda] matrix, K columns.
// Epilogue per element: v = alpha*acc + bias[col] (+ res[row][col]); act; optional tf32 RN.
struct TcGemmArgs {
  int a_mode = 0;
  const float* x = nullptr;
  int n = 0, h = 0, w = 0, cpad = 0;
  int kh = 1, kw = 1, sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1, oh = 0, ow = 0;
  int M = 0, K = 0, lda = 0;
  const float* wt = nullptr;
  int kpad = 0;
  int N = 0;
  const float* bias = nullptr;
  const float* res = nullptr;
  int ldr = 0;
  float* y = nullptr;
  int ldy = 0;
  float alpha = 1.0f;
  int act = 0;
  int round_out = 0;
  int bn = 0;  // 0 = choose
  // Batched GEMM (tiled A only): `batch` problems whose A, Y (and W when b_batched) planes are
  // stored back to back ([batch][M][lda], [batch][M][ldy], [batch][N][kpad]); one launch.
  int batch = 1;
  int b_batched = 0;
  // Visit the tiles from the last one: a planner alternates the direction between consecutive
  // layers so that each starts on the rows its producer wrote last, which are still in L2.
  int reverse = 0;
  int* err = nullptr;  // device error word; nullptr = the per-device flag
  // Split-K workspace (optional).  With one, problems that leave SMs idle are split along K
  // into raw fp32 partials (ksplit x M x N floats) reduced in a fixed order by a finish kernel
  // that applies the epilogue; results stay deterministic.
  float* ws = nullptr;
  size_t ws_bytes = 0;
  // A as the channel concatenation of up to four NHWC tensors (nparts > 1; x unused): part i
  // holds channels [part_c0[i], part_c0[i] + part_cpad[i]) of cpad (im2col) or of K (tiled),
  // each a whole number of channel blocks, stored with its own channel stride part_cpad[i].
  int nparts = 1;
  const float* xpart[4] = {nullptr, nullptr, nullptr, nullptr};
  int part_c0[4] = {0, 0, 0, 0};
  int part_cpad[4] = {0, 0, 0, 0};
  // Stream-K schedule allowed (sk = 1; the planner decides): each CTA (pair) takes an equal
  // share of the problem's k-blocks across tile boundaries, so a short last wave does not
  // idle SMs.  A tile split between CTAs is finished by the CTA holding its first k-blocks,
  // which adds the other CTAs' partial sums (left in `ws`, one slot per CTA) in k order after a
  // bounded wait on their flags.  `sk_flags`: kTcSkFlags zero-initialised ints that only these
  // launches use (each consumer clears the flags it read); launches sharing them must not
  // overlap on the GPU.
  int sk = 0;
  int* sk_flags = nullptr;
};
constexpr int kTcSkFlags = 512;

// Stream-K work split, shared by the kernel and the host-side checks.  Worker w of G owns
// k-blocks [w T / G, (w + 1) T / G) of the T = num_tiles x num_kb k-blocks laid out tile after
// tile (T >= G: every range is non-empty).  Piece i of a worker is its part [kb0, kb1) of
// tile t0 + i; kind 0 is a whole tile, 1 a tail piece (the range starts inside the tile: only
// ever a worker's first piece), 2 the head of a tile that later workers finish (only ever its
// last piece).
struct SkRange {
  long long r0, r1, total;
  int t0, num_kb, workers;
};
__host__ __device__ inline SkRange sk_range(int num_tiles, int num_kb, int w, int workers) {
  SkRange r;
  r.total = (long long)num_tiles * num_kb;
  r.r0 = r.total * w / workers;
  r.r1 = r.total * (w + 1) / workers;
  r.t0 = (int)(r.r0 / num_kb);
  r.num_kb = num_kb;
  r.workers = workers;
  return r;
}
__host__ __device__ inline bool sk_piece(const SkRange& r, int i, int* t, int* kb0, int* kb1, int* kind) {
  *t = r.t0 + i;
  const long long base = (long long)*t * r.num_kb;
  const long long g0 = r.r0 > base ? r.r0 : base;
  const long long g1 = r.r1 < base + r.num_kb ? r.r1 : base + r.num_kb;
  if (g0 >= g1) return false;
  *kb0 = (int)(g0 - base);
  *kb1 = (int)(g1 - base);
  *kind = *kb0 > 0 ? 1 : *kb1 < r.num_kb ? 2 : 0;
  return true;
}
// Whether worker j (> the tile's head worker) holds a tail piece of tile t: its range starts
// before the tile's end.  The contributors of a head piece are the workers after its own
// for which this holds, in order.
__host__ __device__ inline bool sk_contributes(const SkRange& r, int j, int t) {
  return j < r.workers && r.total * j / r.workers < (long long)(t + 1) * r.num_kb;
}
// Workspace a launch of `a` would use (0 when it would not split), for planners.
size_t tc_gemm_workspace_bytes(const TcGemmArgs& a);
// Checks whether the tcgen05 path accepts the problem (alignment, corner ranges ...).
bool tc_gemm_supported(const TcGemmArgs& a, std::string* why);
int tc_gemm_launch(const TcGemmArgs& a, cudaStream_t stream);
// One-warp kernel whose bounded wait on a stream-K flag that nothing raises expires after
// timeout_ns (<= 1 s) and raises *err.
int launch_flag_wait_selftest(int* err, uint64_t timeout_ns, cudaStream_t s);
// Launches so far (process-wide) that ran the stream-K schedule.
uint64_t tc_gemm_streamk_launches();
// The tile plan a launch of this problem would use on `sms` SMs (no workspace limit below the
// launcher's cap): {bn, pair, bk, ms, wr, ksplit, sk}.  Host-only; for checks of the planner.
void tc_gemm_plan_for(int M, int N, int K, int cb, bool has_res, int sms, int taps, bool allow_sk, int out[7]);
// Number of K blocks (32 wide) and padded K the weight matrix must have.
inline int tc_num_kb(int K) { return (K + 31) / 32; }

// ------------------------------------------------------------------ bottleneck tail (tail.cu)
// One launch for a 1x1 expand with a fused residual followed by a 1x1 reduce of its output:
//   y = act_e(t2 * W3^T + b3 + x),  t = act_r(y * W1^T + b1)
// over M rows (pixels, NHWC), t2 [M][k1], x and y [M][n1], t [M][n2]; weights K-major
// W3 [n1][kpad3], W1 [n2][kpad1] (tf32-rounded), act_e 4 (+residual) or 5 (+residual, ReLU),
// act_r 0 or 1 (ReLU).  y is written once and reused from shared memory by the reduce.
struct TailArgs {
  const float* t2 = nullptr;
  const float* x = nullptr;
  const float* w3 = nullptr;
  const float* b3 = nullptr;
  const float* w1 = nullptr;
  const float* b1 = nullptr;
  float* y = nullptr;
  float* t = nullptr;
  int M = 0, k1 = 0, n1 = 0, n2 = 0, kpad3 = 0, kpad1 = 0;
  int act_e = 5, act_r = 1, round_out = 1;
  int* err = nullptr;  // device error word; nullptr = the per-device flag
};
bool tail_fused_supported(const TailArgs& a, std::string* why);
int tail_fused_launch(const TailArgs& a, cudaStream_t stream);

// ------------------------------------------------------------------ Winograd F(4x4,3x3) (winograd.cu)
// 3x3 stride-1 convolution of NHWC x[n][h][w][cpad] into y[n][oh][ow][ocpad] through the
// transform buffers v [36][tiles][3*cpad] and m [36][tiles][ocpad]
// (tiles = n*ceil(oh/4)*ceil(ow/4)) and transformed weights u [36][ocpad][kpad],
// kpad = 32-multiple >= 3*cpad (winograd_f43_weights; split-tf32 products).
struct WinogradArgs {
  const float* x = nullptr;
  int n = 0, h = 0, w = 0, cpad = 0, oh = 0, ow = 0, ph = 1, pw = 1;
  const float* u = nullptr;
  int ocpad = 0, kpad = 0;
  float* v = nullptr;
  float* m = nullptr;
  const float* bias = nullptr;
  const float* res = nullptr;
  float* y = nullptr;
  int act = 0, round_out = 0;
};
inline long winograd_tiles(int n, int oh, int ow) { return (long)n * ((oh + 3) / 4) * ((ow + 3) / 4); }
void winograd_f43_weights(const float* w, int oc, int c, int cpad, int ocpad, int kpad, float* u);
int winograd_f43_run(const WinogradArgs& a, cudaStream_t s);

// ------------------------------------------------------------------ glue kernels (glue.cu)
// round_tf32: round values to tf32 (nearest, ties away) on the way, for tensors that feed an
// MMA operand (the tensor core would otherwise truncate them, a bias that compounds over layers).
int launch_nchw_to_nhwc(const float* x, float* y, int n, int c, int h, int w, int cpad, cudaStream_t s,
                        int round_tf32 = 0);
// NCHW x[n][c][h][w] (c <= 4) -> space-to-depth-2 NHWC y[n][h2][w2][16] with
// y[..][(dy*2+dx)*4 + ch] = x[n][ch][2i+dy-ph][2j+dx-pw] (zero outside / for ch >= c).
int launch_space_to_depth2(const float* x, float* y, int n, int c, int h, int w, int h2, int w2, int ph, int pw,
                           cudaStream_t s, int round_tf32 = 0);
int launch_nhwc_to_nchw(const float* x, float* y, int n, int c, int h, int w, int cpad, cudaStream_t s);
int launch_maxpool_nhwc(const float* x, float* y, int n, int h, int w, int cpad, int oh, int ow, int kh,
                        int kw, int sh, int sw, int ph, int pw, cudaStream_t s);
int launch_avgpool_nhwc(const float* x, float* y, int n, int h, int w, int cpad, int oh, int ow, int kh,
                        int kw, int sh, int sw, int ph, int pw, int count_include_pad, cudaStream_t s);
int launch_gap_nhwc(const float* x, float* y, int n, int hw, int cpad, cudaStream_t s, int round_tf32 = 0);
// y = op(a, b) elementwise with modulo broadcast (SPINN/run_time/ops/math/add.c:4-22).
enum EltOp { ELT_ADD = 0, ELT_MUL = 1, ELT_SUB = 2, ELT_DIV = 3 };
int launch_binary(const float* a, long na, const float* b, long nb, float* y, long n, int op, int act,
                  cudaStream_t s);
enum UnaryOp { UN_RELU = 0, UN_SIGMOID = 1, UN_SILU = 2, UN_COPY = 3 };
int launch_unary(const float* x, float* y, long n, int op, cudaStream_t s);
// Per-channel affine on NHWC: y = x*scale[c] + shift[c] (standalone BatchNormalization).
int launch_channel_affine_nhwc(const float* x, float* y, long pixels, int cpad, const float* scale,
                               const float* shift, cudaStream_t s);
// Depthwise (group == C == OC) and generic grouped direct convolution on NHWC, CUDA cores.
// w layout: [kh*kw][oc] for depthwise; [oc][kh][kw][c/group] for grouped.
int launch_depthwise_nhwc(const float* x, const float* w, const float* bias, const float* res, float* y,
                          int n, int h, int wd, int cpad, int oh, int ow, int kh, int kw, int sh, int sw,
                          int ph, int pw, int dh, int dw, int act, int round_out, cudaStream_t s);
int launch_grouped_nhwc(const float* x, const float* w, const float* bias, const float* res, float* y,
                        int n, int h, int wd, int c, int cpad, int oh, int ow, int oc, int ocpad, int kh,
                        int kw, int sh, int sw, int ph, int pw, int dh, int dw, int group, int act,
                        int round_out, cudaStream_t s);
// Nearest resize, NHWC: y[b][oy][ox] = x[b][oy*h/oh][ox*w/ow] (integer mapping of
// SPINN/run_time/ops/tensor/resize.c:21-30).
int launch_resize_nearest_nhwc(const float* x, float* y, int n, int h, int w, int cpad, int oh, int ow,
                               cudaStream_t s);
// General row-major permutation (ONNX Transpose), up to 8 dimensions: y = x.transpose(perm).
int launch_permute(const float* x, float* y, int ndim, const uint32_t* dims, const uint8_t* perm, cudaStream_t s);
// Softmax over the middle axis of [outer][dim][inner] (SPINN/run_time/ops/activation/softmax.c).
int launch_softmax(const float* x, float* y, long outer, int dim, long inner, cudaStream_t s);
// Row-major transpose of `batch` matrices [rows][cols] -> [cols][rows].
int launch_transpose(const float* x, float* y, int batch, int rows, int cols, cudaStream_t s);
// Split-tf32 packing of a row-major [rows][cols] matrix (leading dimension src_ld) into
// dst rows of dst_ld >= 3*seg floats (seg >= cols): segments in `order` (0 = hi, 1 = lo), hi = tf32(v),
// lo = tf32(v - hi).  With A' = (hi, lo, hi) and B' = (hi, hi, lo), one GEMM over 3*seg gives
// A_hi B_hi + A_lo B_hi + A_hi B_lo.  Only the first `cols` entries of each segment are written.
int launch_split_tf32(const float* src, float* dst, long rows, int cols, int src_ld, int seg, int dst_ld, int o0,
                      int o1, int o2, cudaStream_t s);
// dst[r][0..fill_to) = src[r][0..width) followed by zeros, for r < rows (pitches in floats).
int launch_copy_rows(const float* src, int src_ld, float* dst, int dst_ld, long rows, int width, int fill_to,
                     cudaStream_t s);
// Concat parts along the row-contiguous axis in one launch (offsets, widths multiples of 4).
constexpr int kCatMaxParts = 8;
struct CatParts {
  int n;
  const float* src[kCatMaxParts];
  int ld[kCatMaxParts], off[kCatMaxParts], width[kCatMaxParts];
};
int launch_concat_rows(const CatParts& parts, float* dst, int dst_ld, long rows, int fill_to, cudaStream_t s);
// Split of a row-contiguous axis into dense parts (each part's pitch = its width, widths
// multiples of 4, consecutive offsets) in one launch.
struct SplitParts {
  int n;
  float* dst[kCatMaxParts];
  int ld[kCatMaxParts], off[kCatMaxParts], width[kCatMaxParts];
};
int launch_split_rows(const SplitParts& parts, const float* src, int src_ld, long rows, cudaStream_t s);
// Concat along the last axis of 3-D row-major parts [N][C][L_i] into dst [N][ctot][ltot], where
// a part is given as pieces: channel ranges stored row-major ([N][chans][ld], nhwc = 0) or as
// an NHWC tensor whose H x W positions are the part's L axis ([N][L][ld], channels c0.. of ld;
// nhwc = 1), which is read transposed -- the NCHW conversion of a Reshape [N,C,H,W] -> [N,C,HW]
// and any channel Concat before it happen in this one pass.
constexpr int kGatherMaxPieces = 16;
struct GatherPieces {
  int n;
  const float* src[kGatherMaxPieces];
  int nhwc[kGatherMaxPieces], ld[kGatherMaxPieces], c0[kGatherMaxPieces];
  int chans[kGatherMaxPieces], len[kGatherMaxPieces];
  int dst_c[kGatherMaxPieces], dst_l[kGatherMaxPieces];
};
int launch_gather_rows(const GatherPieces& g, float* dst, int n, int ctot, int ltot, cudaStream_t s);
// TopK over the last axis of a row-major [rows][n] tensor (n <= kTopkMaxN): k largest values
// (descending, ties by ascending index) and their int64 indices, each [rows][k].
constexpr int kTopkMaxN = 16384;
int launch_topk(const float* x, long rows, int n, int k, float* vals, int64_t* idx, cudaStream_t s);
// tf32 round-to-nearest-away in place (weights).
int launch_round_tf32(float* x, long n, cudaStream_t s);

// Host-side tf32 RN (ties away), same rounding as cvt.rna.tf32.f32.
inline float host_round_tf32(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;
  std::memcpy(&f, &u, 4);
  return f;
}

}  // namespace spinn
