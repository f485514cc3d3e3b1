/*
 * spinn_oracle.c -- plain-C restatement of SPINN's dense-contraction hot path.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg as the checker.  Nothing in spinn_b200 links or calls it.
 *
 * Every routine restates the reference operator it names (file:line in the tzp11/spinn
 * tree), in NCHW fp32 with fp32 accumulation, in straightforward loop order (no packing,
 * no SIMD).  It is pinned against the reference objects themselves (oracle/_ref) and
 * against the known-answer inputs of SPINN/run_time/test_winograd*.c in
 * tests/test_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Post-op codes of ENNF_ConvParams.reserved (SPINN/graph_opt.h:31-36). */
enum { ACT_NONE = 0, ACT_RELU = 1, ACT_SILU = 3, ACT_ADD = 4, ACT_ADD_RELU = 5 };

/* Epilogue of sgemm_nn (SPINN/run_time/ops/mm/gemm_kernel.c:316-338). */
static inline float epilogue(float v, float b, const float *res, int act) {
    v += b;
    if (res && (act == ACT_ADD || act == ACT_ADD_RELU)) v += *res;
    if (act == ACT_RELU || act == ACT_ADD_RELU) {
        if (v < 0.0f) v = 0.0f;
    } else if (act == ACT_SILU) {
        v = v / (1.0f + expf(-v));
    }
    return v;
}

/*
 * op_conv2d (SPINN/run_time/ops/conv/conv2d.c:92-232): 2-D convolution, NCHW.
 * Pads are the symmetric pair (pads[0], pads[1]) the reference reads (:131); SAME
 * auto_pad resolved by the caller exactly as :134-141.  Weights [OC][C/group][KH][KW].
 * The K dimension is c-major then kh, kw (im2col row order, :60-77).
 */
int oracle_conv2d(const float *X, int N, int C, int H, int W, const float *Wt, int OC, int KH,
                  int KW, int SH, int SW, int PH, int PW, int DH, int DW, int group,
                  const float *bias, int act, const float *residual, float *Y, int OH, int OW) {
    if (group < 1 || C % group || OC % group) return -1;
    const int KC = C / group, OCg = OC / group;
    const long ohw = (long)OH * OW;
    for (int n = 0; n < N; n++) {
#pragma omp parallel for schedule(static)
        for (int oc = 0; oc < OC; oc++) {
            const int g = oc / OCg;
            const float *w = Wt + (long)oc * KC * KH * KW;
            float *y = Y + ((long)n * OC + oc) * ohw;
            const float *r = residual ? residual + ((long)n * OC + oc) * ohw : NULL;
            for (int oh = 0; oh < OH; oh++) {
                for (int ow = 0; ow < OW; ow++) {
                    float acc = 0.0f;
                    for (int c = 0; c < KC; c++) {
                        const float *x = X + (((long)n * C + g * KC + c) * H) * W;
                        for (int kh = 0; kh < KH; kh++) {
                            const int ih = oh * SH - PH + kh * DH;
                            if (ih < 0 || ih >= H) continue;
                            for (int kw = 0; kw < KW; kw++) {
                                const int iw = ow * SW - PW + kw * DW;
                                if (iw < 0 || iw >= W) continue;
                                acc += w[(c * KH + kh) * KW + kw] * x[(long)ih * W + iw];
                            }
                        }
                    }
                    const long o = (long)oh * OW + ow;
                    y[o] = epilogue(acc, bias ? bias[oc] : 0.0f, r ? r + o : NULL, act);
                }
            }
        }
    }
    return 0;
}

/*
 * op_gemm (SPINN/run_time/ops/mm/gemm.c:7-78) with ONNX semantics
 * Y = alpha * op(A) op(B) + beta * C, C a length-N vector or a full MxN matrix.
 * ref_alpha_quirk=1 reproduces the reference for M>1: sgemm_tiled scales the beta*C
 * pre-fill by alpha as well (gemm.c:62-69 + gemm_kernel.c:298-301), giving
 * alpha*(A B + beta*C); M==1 takes the GEMV path (gemm_kernel.c:215-241) which is exact.
 */
int oracle_gemm(const float *A, const float *B, const float *Cb, long c_elems, float *Y, int M,
                int N, int K, int transA, int transB, float alpha, float beta,
                int ref_alpha_quirk) {
    const int vec = Cb && c_elems == N;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        for (int n = 0; n < N; n++) {
            float acc = 0.0f;
            for (int k = 0; k < K; k++) {
                const float a = transA ? A[(long)k * M + m] : A[(long)m * K + k];
                const float b = transB ? B[(long)n * K + k] : B[(long)k * N + n];
                acc += a * b;
            }
            float c = 0.0f;
            if (Cb && beta != 0.0f) c = beta * Cb[vec ? n : (long)m * N + n];
            float v;
            if (ref_alpha_quirk && M > 1)
                v = alpha * (acc + c);
            else
                v = alpha * acc + c;
            Y[(long)m * N + n] = v;
        }
    }
    return 0;
}

/*
 * op_matmul (SPINN/run_time/ops/mm/matmul.c:6-62): 2-D, batched A with a broadcast 2-D B
 * (:32-44), or equal batch counts (:48-61).  b_batch = 0 means B is 2-D.
 */
int oracle_matmul(const float *A, const float *B, float *Y, int batch, int b_batch, int M, int N,
                  int K) {
    if (b_batch != 0 && b_batch != batch) return -1;
    for (int bi = 0; bi < batch; bi++) {
        const float *a = A + (long)bi * M * K;
        const float *b = B + (b_batch ? (long)bi * K * N : 0);
        float *y = Y + (long)bi * M * N;
#pragma omp parallel for schedule(static)
        for (int m = 0; m < M; m++)
            for (int n = 0; n < N; n++) {
                float acc = 0.0f;
                for (int k = 0; k < K; k++) acc += a[(long)m * K + k] * b[(long)k * N + n];
                y[(long)m * N + n] = acc;
            }
    }
    return 0;
}

/* ---------------- Winograd F(2x2,3x3) (SPINN/run_time/ops/conv/winograd.c) ---------------- */

/* U = G g G^T (winograd.c:40-55). */
static void f23_weight(const float g[3][3], float U[4][4]) {
    float t[4][3];
    for (int j = 0; j < 3; j++) {
        t[0][j] = g[0][j];
        t[1][j] = 0.5f * (g[0][j] + g[1][j] + g[2][j]);
        t[2][j] = 0.5f * (g[0][j] - g[1][j] + g[2][j]);
        t[3][j] = g[2][j];
    }
    for (int i = 0; i < 4; i++) {
        U[i][0] = t[i][0];
        U[i][1] = 0.5f * (t[i][0] + t[i][1] + t[i][2]);
        U[i][2] = 0.5f * (t[i][0] - t[i][1] + t[i][2]);
        U[i][3] = t[i][2];
    }
}

/* V = B^T d B (winograd.c:23-37). */
static void f23_input(const float d[4][4], float V[4][4]) {
    float t[4][4];
    for (int j = 0; j < 4; j++) {
        t[0][j] = d[0][j] - d[2][j];
        t[1][j] = d[1][j] + d[2][j];
        t[2][j] = -d[1][j] + d[2][j];
        t[3][j] = d[1][j] - d[3][j];
    }
    for (int i = 0; i < 4; i++) {
        V[i][0] = t[i][0] - t[i][2];
        V[i][1] = t[i][1] + t[i][2];
        V[i][2] = -t[i][1] + t[i][2];
        V[i][3] = t[i][1] - t[i][3];
    }
}

/* Y = A^T M A (winograd.c:57-67). */
static void f23_output(const float M[4][4], float o[2][2]) {
    float t[2][4];
    for (int j = 0; j < 4; j++) {
        t[0][j] = M[0][j] + M[1][j] + M[2][j];
        t[1][j] = M[1][j] - M[2][j] - M[3][j];
    }
    for (int i = 0; i < 2; i++) {
        o[i][0] = t[i][0] + t[i][1] + t[i][2];
        o[i][1] = t[i][1] - t[i][2] - t[i][3];
    }
}

/* winograd_pack_weight (winograd.c:70-90): U laid out [16][OC*C]. */
void oracle_winograd_f23_pack(const float *Wt, int OC, int C, float *U) {
    for (int oc = 0; oc < OC; oc++)
        for (int c = 0; c < C; c++) {
            float g[3][3], u[4][4];
            for (int i = 0; i < 9; i++) g[i / 3][i % 3] = Wt[((long)oc * C + c) * 9 + i];
            f23_weight(g, u);
            for (int a = 0; a < 16; a++) U[(long)a * OC * C + (long)oc * C + c] = u[a / 4][a % 4];
        }
}

/*
 * winograd_conv_3x3 (winograd.c:96-210): 2x2 output tiles, 16 transform-domain GEMMs,
 * bias, and ReLU when fused_relu != 0 (any non-zero code, :200).  Returns -1 for fewer
 * than 4 tiles or a workspace above 64M floats (:107-111), as the reference does.
 */
int oracle_winograd_f23(const float *X, int N, int C, int H, int W, const float *U, int OC,
                        const float *bias, int PH, int PW, float *Y, int OH, int OW, int fused_relu) {
    const int th = (OH + 1) / 2, tw = (OW + 1) / 2, nt = th * tw;
    if (nt < 4) return -1;
    if ((size_t)16 * C * nt + (size_t)16 * OC * nt > (size_t)64 * 1024 * 1024) return -1;
    float *V = (float *)calloc((size_t)16 * C * nt, sizeof(float));
    float *Mo = (float *)calloc((size_t)16 * OC * nt, sizeof(float));
    if (!V || !Mo) { free(V); free(Mo); return -1; }
    for (int n = 0; n < N; n++) {
        const float *Xn = X + (long)n * C * H * W;
        float *Yn = Y + (long)n * OC * OH * OW;
        for (int c = 0; c < C; c++)
            for (int ti = 0; ti < th; ti++)
                for (int tj = 0; tj < tw; tj++) {
                    float d[4][4], v[4][4];
                    for (int i = 0; i < 4; i++)
                        for (int j = 0; j < 4; j++) {
                            int ih = ti * 2 + i - PH, iw = tj * 2 + j - PW;
                            d[i][j] = (ih >= 0 && ih < H && iw >= 0 && iw < W) ? Xn[((long)c * H + ih) * W + iw] : 0.0f;
                        }
                    f23_input(d, v);
                    for (int a = 0; a < 16; a++) V[(long)a * C * nt + (long)c * nt + ti * tw + tj] = v[a / 4][a % 4];
                }
        for (int a = 0; a < 16; a++)
#pragma omp parallel for schedule(static)
            for (int oc = 0; oc < OC; oc++)
                for (int t = 0; t < nt; t++) {
                    float acc = 0.0f;
                    for (int c = 0; c < C; c++) acc += U[(long)a * OC * C + (long)oc * C + c] * V[(long)a * C * nt + (long)c * nt + t];
                    Mo[(long)a * OC * nt + (long)oc * nt + t] = acc;
                }
        for (int oc = 0; oc < OC; oc++)
            for (int ti = 0; ti < th; ti++)
                for (int tj = 0; tj < tw; tj++) {
                    float m[4][4], o[2][2];
                    for (int a = 0; a < 16; a++) m[a / 4][a % 4] = Mo[(long)a * OC * nt + (long)oc * nt + ti * tw + tj];
                    f23_output(m, o);
                    for (int i = 0; i < 2 && ti * 2 + i < OH; i++)
                        for (int j = 0; j < 2 && tj * 2 + j < OW; j++) {
                            float v = o[i][j] + (bias ? bias[oc] : 0.0f);
                            if (fused_relu && v < 0.0f) v = 0.0f;
                            Yn[((long)oc * OH + ti * 2 + i) * OW + tj * 2 + j] = v;
                        }
                }
    }
    free(V);
    free(Mo);
    return 0;
}

/* ---------------- Winograd F(4x4,3x3) (new; no reference implementation) ----------------
 * Lavin & Gray 2016 transforms with interpolation points {0, 1, -1, 2, -2, inf}:
 *   B^T = [4 0 -5 0 1 0; 0 -4 -4 1 1 0; 0 4 -4 -1 1 0; 0 -2 -1 2 1 0; 0 2 -1 -2 1 0; 0 4 0 -5 0 1]
 *   G   = [1/4 0 0; -1/6 -1/6 -1/6; -1/6 1/6 -1/6; 1/24 1/12 1/6; 1/24 -1/12 1/6; 0 0 1]
 *   A^T = [1 1 1 1 1 0; 0 1 -1 2 -2 0; 0 1 1 4 4 0; 0 1 -1 8 -8 1]
 * Same structure as the F(2,3) routine above (transform, per-point GEMM, inverse
 * transform + epilogue), computed in double so that it serves as a structure check of
 * the device transforms; the fused post-op follows sgemm_nn (all act codes). */
static const double F43_BT[6][6] = {{4, 0, -5, 0, 1, 0},  {0, -4, -4, 1, 1, 0}, {0, 4, -4, -1, 1, 0},
                                    {0, -2, -1, 2, 1, 0}, {0, 2, -1, -2, 1, 0}, {0, 4, 0, -5, 0, 1}};
static const double F43_G[6][3] = {{1.0 / 4, 0, 0},           {-1.0 / 6, -1.0 / 6, -1.0 / 6},
                                   {-1.0 / 6, 1.0 / 6, -1.0 / 6}, {1.0 / 24, 1.0 / 12, 1.0 / 6},
                                   {1.0 / 24, -1.0 / 12, 1.0 / 6}, {0, 0, 1}};
static const double F43_AT[4][6] = {{1, 1, 1, 1, 1, 0}, {0, 1, -1, 2, -2, 0}, {0, 1, 1, 4, 4, 0}, {0, 1, -1, 8, -8, 1}};

/* U[36][OC][C] = G g G^T, stored as float. */
void oracle_winograd_f43_pack(const float *Wt, int OC, int C, float *U) {
    for (int oc = 0; oc < OC; oc++)
        for (int c = 0; c < C; c++) {
            const float *g = Wt + ((long)oc * C + c) * 9;
            double t[6][3];
            for (int i = 0; i < 6; i++)
                for (int j = 0; j < 3; j++)
                    t[i][j] = F43_G[i][0] * g[0 * 3 + j] + F43_G[i][1] * g[1 * 3 + j] + F43_G[i][2] * g[2 * 3 + j];
            for (int i = 0; i < 6; i++)
                for (int j = 0; j < 6; j++) {
                    double u = t[i][0] * F43_G[j][0] + t[i][1] * F43_G[j][1] + t[i][2] * F43_G[j][2];
                    U[((long)(i * 6 + j) * OC + oc) * C + c] = (float)u;
                }
        }
}

/* 3x3 stride-1 convolution through F(4x4,3x3) with pad (PH, PW), NCHW. */
int oracle_winograd_f43(const float *X, int N, int C, int H, int W, const float *U, int OC,
                        const float *bias, int act, const float *residual, int PH, int PW,
                        float *Y, int OH, int OW) {
    const int th = (OH + 3) / 4, tw = (OW + 3) / 4, nt = th * tw;
    double *V = (double *)malloc(sizeof(double) * 36 * (size_t)C * nt);
    if (!V) return -1;
    for (int n = 0; n < N; n++) {
        const float *Xn = X + (long)n * C * H * W;
#pragma omp parallel for schedule(static)
        for (int c = 0; c < C; c++)
            for (int t = 0; t < nt; t++) {
                const int ti = t / tw, tj = t % tw;
                double d[6][6], tmp[6][6];
                for (int i = 0; i < 6; i++)
                    for (int j = 0; j < 6; j++) {
                        int ih = ti * 4 + i - PH, iw = tj * 4 + j - PW;
                        d[i][j] = (ih >= 0 && ih < H && iw >= 0 && iw < W) ? Xn[((long)c * H + ih) * W + iw] : 0.0;
                    }
                for (int i = 0; i < 6; i++)
                    for (int j = 0; j < 6; j++) {
                        double s = 0;
                        for (int k = 0; k < 6; k++) s += F43_BT[i][k] * d[k][j];
                        tmp[i][j] = s;
                    }
                for (int i = 0; i < 6; i++)
                    for (int j = 0; j < 6; j++) {
                        double s = 0;
                        for (int k = 0; k < 6; k++) s += tmp[i][k] * F43_BT[j][k];
                        V[((long)(i * 6 + j) * C + c) * nt + t] = s;
                    }
            }
#pragma omp parallel for schedule(static)
        for (int oc = 0; oc < OC; oc++) {
            double *Mt = (double *)malloc(sizeof(double) * 36 * nt);
            for (int a = 0; a < 36; a++)
                for (int t = 0; t < nt; t++) {
                    double s = 0;
                    for (int c = 0; c < C; c++) s += (double)U[((long)a * OC + oc) * C + c] * V[((long)a * C + c) * nt + t];
                    Mt[(long)a * nt + t] = s;
                }
            for (int t = 0; t < nt; t++) {
                const int ti = t / tw, tj = t % tw;
                double tmp[4][6];
                for (int i = 0; i < 4; i++)
                    for (int j = 0; j < 6; j++) {
                        double s = 0;
                        for (int k = 0; k < 6; k++) s += F43_AT[i][k] * Mt[(long)(k * 6 + j) * nt + t];
                        tmp[i][j] = s;
                    }
                for (int i = 0; i < 4; i++)
                    for (int j = 0; j < 4; j++) {
                        const int oh = ti * 4 + i, ow = tj * 4 + j;
                        if (oh >= OH || ow >= OW) continue;
                        double s = 0;
                        for (int k = 0; k < 6; k++) s += tmp[i][k] * F43_AT[j][k];
                        const long o = (((long)n * OC + oc) * OH + oh) * OW + ow;
                        Y[o] = epilogue((float)s, bias ? bias[oc] : 0.0f, residual ? residual + o : NULL, act);
                    }
            }
            free(Mt);
        }
    }
    free(V);
    return 0;
}

/* ---------------- glue operators on the ResNet/YOLO graphs ---------------- */

/* op_maxpool (SPINN/run_time/ops/pool/maxpool.c:5-49): pads (pads[0], pads[1]); -1e30 init. */
int oracle_maxpool(const float *X, int N, int C, int H, int W, int KH, int KW, int SH, int SW,
                   int PH, int PW, float *Y, int OH, int OW) {
#pragma omp parallel for schedule(static)
    for (long nc = 0; nc < (long)N * C; nc++)
        for (int oh = 0; oh < OH; oh++)
            for (int ow = 0; ow < OW; ow++) {
                float m = -1e30f;
                for (int kh = 0; kh < KH; kh++)
                    for (int kw = 0; kw < KW; kw++) {
                        int ih = oh * SH - PH + kh, iw = ow * SW - PW + kw;
                        if (ih >= 0 && ih < H && iw >= 0 && iw < W) {
                            float v = X[(nc * H + ih) * W + iw];
                            if (v > m) m = v;
                        }
                    }
                Y[(nc * OH + oh) * OW + ow] = m;
            }
    return 0;
}

/* op_global_avg_pool (SPINN/run_time/ops/pool/global_avg_pool.c:4-28): fp32 sum / HW. */
int oracle_global_avg_pool(const float *X, int N, int C, int HW, float *Y) {
    for (long nc = 0; nc < (long)N * C; nc++) {
        float s = 0.0f;
        for (int i = 0; i < HW; i++) s += X[nc * HW + i];
        Y[nc] = s / HW;
    }
    return 0;
}

/* op_add (SPINN/run_time/ops/math/add.c:4-22): modulo broadcast. */
int oracle_add(const float *a, long na, const float *b, long nb, float *y, long n) {
    for (long i = 0; i < n; i++) y[i] = a[i % na] + b[i % nb];
    return 0;
}

/* op_relu (SPINN/run_time/ops/activation/relu.c:4-18). */
int oracle_relu(const float *x, float *y, long n) {
    for (long i = 0; i < n; i++) y[i] = x[i] > 0 ? x[i] : 0;
    return 0;
}

/* op_sigmoid on scalars, 1/(1+exp(-x)). */
int oracle_sigmoid(const float *x, float *y, long n) {
    for (long i = 0; i < n; i++) y[i] = 1.0f / (1.0f + expf(-x[i]));
    return 0;
}

/* op_batch_norm (SPINN/run_time/ops/norm/batch_norm.c:17-76): alpha = g/sqrt(v+eps),
 * beta' = b - m*alpha, y = x*alpha + beta'. */
int oracle_batch_norm(const float *X, int N, int C, int HW, const float *g, const float *b,
                      const float *m, const float *v, float eps, float *Y) {
    for (int c = 0; c < C; c++) {
        const float a = g[c] / sqrtf(v[c] + eps), bb = b[c] - m[c] * a;
        for (int n = 0; n < N; n++)
            for (int i = 0; i < HW; i++) {
                const long o = ((long)n * C + c) * HW + i;
                Y[o] = X[o] * a + bb;
            }
    }
    return 0;
}
