/*
 * spinn_cuda.h -- C ABI of libspinn_cuda.so, the B200 (sm_100a) implementation of SPINN's
 * dense-contraction hot path (Conv / Gemm / MatMul and the Conv+BN/ReLU/SiLU/Add fusions).
 *
 * Two levels, both plain C (pointers, sizes, status codes; no C++ or torch types):
 *
 *  1. Operator level: drop-in replacements for the reference operators, with the
 *     reference's SpinnOpKernel signature, so SPINN's own runtime (spinn_load / spinn_plan /
 *     spinn_run) can dispatch Conv, Gemm and MatMul to the GPU unchanged.  Tensor data may
 *     be host memory (the reference arena) or device memory; results are written where
 *     out[0]->data points.
 *
 *  2. Model level: a device-resident executor for a whole .ennf model that mirrors the
 *     reference's three stages (load -> plan -> run): one device arena, weights uploaded
 *     once and pre-transformed, every node on the GPU, the node list replayed as a CUDA
 *     graph.
 *
 * Every entry point returns 0 on success and a negative SPINN_CUDA_E* code on failure;
 * spinn_cuda_last_error() gives the message of the most recent failure on the calling thread.
 * The reference runtime ignores operator return codes (SPINN/run_time/spinn_runtime.c:331-345);
 * these do not.
 */
#ifndef SPINN_CUDA_H
#define SPINN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ shared types */

/* Runtime tensor record.  Byte-for-byte the reference's SpinnTensor
 * (SPINN/run_time/spinn_runtime.h:25-40): 72 bytes on LP64, `data` at offset 56. */
#define SPINN_CUDA_MAX_DIMS 8
typedef struct {
    uint16_t id;
    uint8_t dtype;
    uint8_t ndim;
    uint32_t dims[SPINN_CUDA_MAX_DIMS];
    uint32_t elem_count;
    uint8_t is_weight;
    uint8_t ref_count;
    uint32_t size;
    uint32_t offset;
    void *data;
    void *packed_data; /* never touched here: the reference runtime free()s it */
} SpinnTensor;

/* Operator kernel signature (SPINN/run_time/spinn_ops.h:31-33). */
typedef int (*SpinnOpKernel)(SpinnTensor **in, int n_in, void *params, uint16_t params_size,
                             SpinnTensor **out, int n_out);

/* Status codes. */
#define SPINN_CUDA_OK 0
#define SPINN_CUDA_EINVAL (-1)     /* bad argument, shape or parameter block */
#define SPINN_CUDA_ENOMEM (-2)     /* device or host allocation failed / arena budget exceeded */
#define SPINN_CUDA_ECUDA (-3)      /* CUDA runtime or driver error */
#define SPINN_CUDA_EUNSUPPORTED (-4) /* operator or configuration not implemented */
#define SPINN_CUDA_ETIMEOUT (-5)   /* a kernel's bounded wait expired (device error flag set) */
#define SPINN_CUDA_EFORMAT (-6)    /* malformed .ennf image */
#define SPINN_CUDA_ESTATE (-7)     /* call out of order (e.g. run before plan) */

/* ------------------------------------------------------------------ device session */

/* Selects `device` for the calling thread, creates its stream and a scratch pool of
 * `scratch_bytes` (0 = grow on demand).  Must precede the operator-level entry points.
 * Replaces nothing in the reference (it has no device); called once per GPU thread. */
int spinn_cuda_init(int device, size_t scratch_bytes);

/* Waits for all work queued by this thread's session; returns the first deferred error. */
int spinn_cuda_sync(void);

/* Diagnostic: runs a one-thread kernel whose bounded mbarrier wait -- the primitive every
 * tcgen05 kernel waits with -- expires after timeout_ns (at most 1 s), and reports it.  Returns
 * SPINN_CUDA_ETIMEOUT when the expiry was detected and cleared (the expected result); the
 * context stays usable. */
int spinn_cuda_selftest_wait_expiry(uint64_t timeout_ns);

/* Diagnostic: the same for the bounded wait on a stream-K handoff flag (acquire loads of a
 * word another CTA raises): one warp waits on a flag nothing raises; SPINN_CUDA_ETIMEOUT is the
 * expected result, the context stays usable. */
int spinn_cuda_selftest_flag_wait_expiry(uint64_t timeout_ns);

/* Releases the calling thread's session (stream, scratch, cached weights). */
void spinn_cuda_shutdown(void);

/* Message of the last failure on this thread ("" if none).  Never NULL. */
const char *spinn_cuda_last_error(void);

/* Installs spinn_cuda_conv2d / _gemm / _matmul into a registry through `register_op`
 * (op_type: ENNF_OpType value; Conv=60, Gemm=160, MatMul=161, SPINN/ennf_op_types.h:79,134,135).
 * The reference registry is a file-static array (SPINN/run_time/spinn_ops.c:17), so the
 * reference needs a one-function setter, e.g. `int spinn_register_op(uint16_t op,
 * SpinnOpKernel fn) { g_op_registry[op] = fn; return 0; }` beside init_registry.
 * Returns the number of operators installed. */
int spinn_cuda_register(int (*register_op)(uint16_t op_type, SpinnOpKernel fn));

/* ------------------------------------------------------------------ operator level */

/* ONNX Conv (2-D, NCHW) with the fused post-op in ENNF_ConvParams.reserved
 * (0 none, 1 ReLU, 3 SiLU, 4 +residual, 5 +residual then ReLU; residual = last input).
 * Replaces op_conv2d (SPINN/run_time/ops/conv/conv2d.c:92-232; declared ops/kernels.h:75).
 * Unlike the reference's group==1 path (gemm_kernel.c:497-590) the fused post-op is applied. */
int spinn_cuda_conv2d(SpinnTensor **in, int n_in, void *params, uint16_t params_size,
                      SpinnTensor **out, int n_out);

/* ONNX Gemm Y = alpha*op(A)*op(B) + beta*C (C: length-N vector or MxN).
 * Replaces op_gemm (SPINN/run_time/ops/mm/gemm.c:7-78; declared ops/kernels.h:80).
 * Implements ONNX semantics for every M; the reference multiplies beta*C by alpha too when
 * M > 1 (gemm.c:62-69 with gemm_kernel.c:298-301). */
int spinn_cuda_gemm(SpinnTensor **in, int n_in, void *params, uint16_t params_size,
                    SpinnTensor **out, int n_out);

/* MatMul: 2-D, batched A with broadcast 2-D B, or equal batch counts.
 * Replaces op_matmul (SPINN/run_time/ops/mm/matmul.c:6-62; declared ops/kernels.h:81). */
int spinn_cuda_matmul(SpinnTensor **in, int n_in, void *params, uint16_t params_size,
                      SpinnTensor **out, int n_out);

/* Convolution that allocates nothing (no counterpart in the reference).  For hosts that must
 * not allocate device memory while running -- SPINN's own deployment model plans all memory
 * up front -- this variant of spinn_cuda_conv2d keeps every temporary in one fixed 32 MiB
 * device array that each GPU loading the library holds until exit.  Arguments are device
 * pointers (NCHW fp32 x, OIHW w, optional bias[oc], residual like y when fused_act is 4/5)
 * and the geometry; group 1.  Refused with SPINN_CUDA_EINVAL before any GPU work: problems
 * whose temporaries exceed the 32 MiB, batch n > 65535, stride > 8, padding that puts the
 * im2col corners outside [-128, 127], and a `stream` of a device other than the current one.
 * The first call on a device resolves the array's address; under lazy module loading (the
 * CUDA default) the first call of each shape also loads kernel code, which allocates, so make
 * those calls during set-up (or set CUDA_MODULE_LOADING=EAGER).  Never call it while its
 * stream, or any stream under a global-mode capture, is capturing: it reads an error word back
 * to the host and waits for `stream` before returning.  Calls overlapping on the GPU share the
 * array and race. */
int spinn_cuda_conv2d_noalloc(const float *x, const float *w, const float *bias, const float *residual,
                              float *y, int n, int c, int h, int w_, int oc, int kh, int kw,
                              int stride_h, int stride_w, int pad_h, int pad_w, int fused_act,
                              void *stream);

/* ------------------------------------------------------------------ model level */

typedef struct SpinnCudaModel SpinnCudaModel;

/* Stage 1: parse a .ennf file / in-memory image (copied).  Mirrors spinn_load
 * (SPINN/run_time/spinn_runtime.h:107-112).  NULL on failure (see spinn_cuda_last_error). */
SpinnCudaModel *spinn_cuda_load(const char *path);
SpinnCudaModel *spinn_cuda_load_buffer(const void *data, size_t size);

/* Stage 2: plan and allocate on `device`: one device arena (64-bit offsets; budget
 * max_arena_bytes, 0 = unlimited), weights uploaded and pre-transformed, kernels chosen.
 * Mirrors spinn_plan (spinn_runtime.h:114-123; SPINN_MEM_ERR_NOMEM -> SPINN_CUDA_ENOMEM).
 * flags: bit 0 = do not capture a CUDA graph; bit 1 = also prepare a profiled variant
 *        (spinn_cuda_run_profiled);
 *        bit 2 = keep activations fp32 on store (no tf32 rounding of conv outputs);
 *        bit 3 = Winograd F(4x4,3x3) for 3x3 stride-1 group-1 convolutions;
 *        bit 4 = keep every intermediate tensor after a run (each gets its own arena range);
 *        bit 5 = no cross-layer fusion.  By default (a) a 1x1 convolution with a fused residual
 *        followed by a 1x1 convolution of its output (a bottleneck block's end and the next
 *        block's start) runs as one kernel when the tensors are large enough: its output is
 *        written once and fed to the second convolution from on-chip memory; (b) a channel
 *        Concat whose only reader is a tensor-core convolution is not materialised: the
 *        convolution fetches each channel block from the Concat's inputs. */
#define SPINN_CUDA_PLAN_NO_GRAPH 1
#define SPINN_CUDA_PLAN_PROFILE 2
#define SPINN_CUDA_PLAN_NO_ROUND 4
#define SPINN_CUDA_PLAN_WINOGRAD 8 /* run 3x3 stride-1 convolutions with Winograd F(4x4,3x3) */
#define SPINN_CUDA_PLAN_KEEP 16    /* keep every intermediate tensor (no arena reuse) for
                                      spinn_cuda_copy_tensor; same kernels and tile plans */
#define SPINN_CUDA_PLAN_NO_FUSE 32 /* no cross-layer fusion (see below) */
int spinn_cuda_plan(SpinnCudaModel *m, int device, uint64_t max_arena_bytes, int flags);

/* Stage 3: run one inference.  Copies input 0 (NCHW fp32, host memory) to the device, runs
 * every node, and copies output 0 back to `output` (host).  Mirrors spinn_run
 * (spinn_runtime.h:125-131).  Synchronous. */
int spinn_cuda_run(SpinnCudaModel *m, const void *input, void *output);

/* Pipelined runs (serving loops): spinn_cuda_submit queues one inference -- input 0 copied
 * from `input` (host, pinned for overlap) on a copy stream into one of two device input
 * buffers (the first submission captures a second graph reading the other one), the run,
 * output 0 copied back to `output` -- and returns without waiting, so the input copy of the
 * next submission overlaps this one's run.  `input` and `output` must stay
 * valid and untouched until spinn_cuda_wait returns; results arrive in submission order.
 * Either pointer may be NULL (no copy).  spinn_cuda_wait blocks until every submitted run has
 * finished and reports a deferred error (a kernel's expired wait: SPINN_CUDA_ETIMEOUT). */
int spinn_cuda_submit(SpinnCudaModel *m, const void *input, void *output);
int spinn_cuda_wait(SpinnCudaModel *m);

/* Device-resident run: inputs are taken from, and outputs left in, the model's device
 * buffers (spinn_cuda_io_ptr); work is queued on `stream` (NULL = the model's stream) and
 * not waited for. */
int spinn_cuda_run_device(SpinnCudaModel *m, void *stream);

/* Profiled run (plan flag PROFILE): the step list with a CUDA event between steps, replayed
 * from its own captured graph; synchronous.  Per-step device times via spinn_cuda_profile. */
int spinn_cuda_run_profiled(SpinnCudaModel *m, void *stream);

/* Device buffer of graph input (is_output=0) or output (is_output=1) number `index`,
 * NCHW fp32 as the .ennf declares it, and its size in bytes. */
void *spinn_cuda_io_ptr(SpinnCudaModel *m, int is_output, int index, size_t *bytes);

/* Number of graph inputs / outputs, and the dims of one (returns ndim, fills dims[8]). */
int spinn_cuda_io_count(SpinnCudaModel *m, int is_output);
int spinn_cuda_io_dims(SpinnCudaModel *m, int is_output, int index, uint32_t *dims);

/* ENNF data type of graph input / output `index` (1 fp32, 7 int64 -- TopK indices keep 8
 * bytes per element on the device), or < 0. */
int spinn_cuda_io_dtype(SpinnCudaModel *m, int is_output, int index);

/* Synchronous copy of graph output `index` (after a run) into host memory; `bytes` must be
 * the output's size (spinn_cuda_io_ptr). */
int spinn_cuda_copy_output(SpinnCudaModel *m, int index, void *host, size_t bytes);

/* Synchronous copy of items [first, first + count) along dim 0 (the images of an NCHW
 * tensor) of ENNF tensor `tensor_id` after a run, in the .ennf's own layout (NCHW fp32 for
 * 4-D tensors), into `host`; `bytes` must be exactly their size.  Graph outputs can always be
 * read; any other activation needs plan flag SPINN_CUDA_PLAN_KEEP (otherwise its arena range
 * has been reused).  Weights and tensors fused away by the converter return EINVAL.  The
 * reference keeps intermediates in its host arena (SPINN/run_time/spinn_runtime.c:147-152);
 * this is how a caller inspects them here, e.g. for per-layer checks. */
int spinn_cuda_copy_tensor(SpinnCudaModel *m, int tensor_id, int first, int count, void *host, size_t bytes);

/* Planned sizes: device arena bytes and pre-transformed weight bytes; the number of steps and
 * the kernels one run launches (the captured graph's kernel nodes; without a graph, the steps
 * that launch a kernel). */
int spinn_cuda_plan_info(SpinnCudaModel *m, uint64_t *arena_bytes, uint64_t *weight_bytes,
                         int *num_steps, int *num_kernels);

/* Per-step device times of the last profiled run: fills up to `cap` entries of
 * op_type / milliseconds / algorithmic FLOPs; returns the number of entries. */
int spinn_cuda_profile(SpinnCudaModel *m, int *op_types, float *ms, double *flops, int cap);

/* Kernel id of step `i` (for reporting): 0 none/alias, 1 tcgen05 conv, 2 tcgen05 gemm,
 * 3 depthwise, 4 direct conv, 5 pool, 6 elementwise, 7 layout, 8 winograd, 9 tcgen05 bottleneck
 * tail (two convolutions in one step). */
int spinn_cuda_step_kind(SpinnCudaModel *m, int i);

/* Stage 4: free everything the model owns.  Mirrors spinn_free (spinn_runtime.h:133). */
void spinn_cuda_free(SpinnCudaModel *m);

/* Page-locked host memory for fast host<->device copies (cudaHostAlloc / cudaFreeHost). */
void *spinn_cuda_host_alloc(size_t bytes);
void spinn_cuda_host_free(void *p);

/* Library version string. */
const char *spinn_cuda_version(void);

/* Diagnostics: tcgen05 launches so far in this process that ran a stream-K schedule (each
 * CTA an equal share of the problem's k-blocks across tile boundaries). */
uint64_t spinn_cuda_stat_streamk_launches(void);

/* Diagnostics (host only, no GPU needed): the tile plan the tcgen05 planner makes for an
 * M x N x K problem with channel blocks of `channel_block` (4/8/16/32) floats, `taps` filter
 * taps (1 for a GEMM), on `sms` SMs: out7 = {tile width, CTA pair (2) or single (1), stage
 * depth, M sub-tiles, resident weights, K split, stream-K}.  SPINN_TC_TILES, when set, applies
 * as it does to launches. */
int spinn_cuda_diag_tile_plan(int m, int n, int k, int channel_block, int has_residual, int sms, int taps,
                              int allow_streamk, int *out7);
/* Diagnostics (host only): piece `piece` of stream-K worker `worker` of `workers` over
 * num_tiles x num_kb k-blocks: returns 1 and out4 = {tile, first k-block, end k-block, kind
 * (0 whole tile, 1 tail part, 2 head part)}, 0 past the worker's last piece, or an error. */
int spinn_cuda_diag_streamk_piece(int num_tiles, int num_kb, int worker, int workers, int piece, int *out4);
/* Diagnostics (host only): 1 when worker `worker` holds a tail part of tile `tile`, judged as
 * the head worker of that tile does (the worker's range starts before the tile's end). */
int spinn_cuda_diag_streamk_contributes(int num_tiles, int num_kb, int worker, int workers, int tile);

#ifdef __cplusplus
}
#endif

#endif /* SPINN_CUDA_H */
