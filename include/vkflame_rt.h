/*
 * vkflame_rt.h — C ABI of libvkflame_rt.so, the B200 runtime under the shims.
 *
 * Replaces the reference's Vulkan runtime (runtime/device.h, runtime/buffer.h,
 * runtime/dispatch.h) with a thin layer over the CUDA runtime.  Pointers are
 * real CUDA device pointers; streams are cudaStream_t (hipStream_t values
 * handed out by libamdhip64 are cudaStream_t); NULL means the legacy default
 * stream.  Every entry point returns a vkflame status (0 = success) and also
 * records it as the calling thread's last error.
 *
 * Entry points that exist in the reference keep its name and argument order
 * (a caller that ignores the return value, as the reference's void functions
 * imply, still links and runs).  Each is annotated with the reference
 * declaration it replaces.
 */
#ifndef VKFLAME_RT_H
#define VKFLAME_RT_H

#include <stddef.h>
#include <stdint.h>
#include "ggml_blocks.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define VKF_OK 0
#define VKF_ERR_INVALID 1      /* bad shape / enum / NULL argument            */
#define VKF_ERR_NOMEM 2        /* device allocation failed                      */
#define VKF_ERR_BADPTR 3       /* pointer not device-accessible / out of range  */
#define VKF_ERR_UNSUPPORTED 4  /* valid request this build does not implement   */
#define VKF_ERR_CUDA 5         /* a CUDA call or kernel launch failed           */
#define VKF_ERR_NO_DEVICE 6    /* no sm_100 device present                      */
#define VKF_ERR_TIMEOUT 7      /* a kernel gave up a bounded wait (see below)   */

/* Dtype codes of vkflame_dispatch_linear (runtime/dispatch.h:7-11). */
#define VKF_DTYPE_FP32 0
#define VKF_DTYPE_FP16 1
#define VKF_DTYPE_INT8 2
#define VKF_DTYPE_BF16 3
#define VKF_DTYPE_FP16_FP32OUT 4

/* Activation codes (kernels/linear_fp16.glsl:19, linear_int8.glsl:23). */
#define VKF_ACT_NONE 0
#define VKF_ACT_SILU 1
#define VKF_ACT_RELU 2
#define VKF_ACT_GELU_ERF 3

/* Activation / output element types of vkflame_quant_linear. */
#define VKF_X_F16 0
#define VKF_X_Q8_1 1
#define VKF_Y_F32 0
#define VKF_Y_F16 1

/* ---- device (runtime/device.h:39-42) ----------------------------------- */
int vkflame_init(void);               /* idempotent; selects/validates the current device */
void *vkflame_get_context(void);      /* opaque, non-NULL after init; never dereferenced by callers */
void vkflame_shutdown(void);
void vkflame_print_info(void);

/* ---- memory (runtime/buffer.h:22-62; VKFBuffer* becomes a device pointer) */
void *vkflame_alloc(size_t size);     /* cudaMalloc + allocation table; NULL on failure */
int vkflame_free(void *ptr);
int vkflame_memcpy_h2d(void *dst, const void *src, size_t size, size_t offset);
int vkflame_memcpy_d2h(void *dst, const void *src, size_t size, size_t offset);
int vkflame_memcpy_d2d(void *dst, const void *src, size_t size);
int vkflame_memset(void *dst, int value, size_t size);
/* Range lookup: any pointer inside a live vkflame_alloc block resolves to
 * its base and size (the reference only matched block bases,
 * shim/hip_runtime_shim.cpp:399-406). Returns VKF_ERR_BADPTR if unknown. */
int vkflame_ptr_lookup(const void *ptr, void **base, size_t *size);
/* Registers an allocation made elsewhere (e.g. by the hip shim) so range
 * checks accept it. */
int vkflame_register_alloc(void *base, size_t size);
int vkflame_unregister_alloc(void *base);

/* ---- dispatch (runtime/dispatch.h:51-92) -------------------------------- */

/* runtime/dispatch.h:51-58.  Row-major D[MxN] = act(alpha * op(A) op(B) + beta * C).
 * A is M x K (transA=1: stored K x M); B is K x N (transB=1: stored N x K).
 * dtype selects element types as VKF_DTYPE_*; FP16_FP32OUT writes fp32 D.
 * alpha/beta are host pointers to scalars of the compute type (fp32 for
 * every dtype here; NULL means 1 and 0). */
int vkflame_dispatch_linear(void *ctx, const void *A, const void *B, const void *C, void *D,
                            int M, int N, int K, int dtype, int transA, int transB,
                            int activation, const void *alpha, const void *beta, void *stream);

/* runtime/dispatch.h:89-92.  Dequantise n_blocks blocks of quant_type to fp32
 * (n_blocks counts blocks of the format: 32 values for Q4_0/Q4_1/Q5_0/Q8_0/Q8_1,
 * 256 for Q4_K/Q5_K/Q6_K).  Bit-exact with kernels/dequant_*.glsl.
 * The reference's src/dst were VKFBuffer*; here they are device pointers,
 * and a sub-allocation offset inside them is honoured. */
int vkflame_dispatch_dequant(void *ctx, const void *src, void *dst, uint32_t n_blocks, int quant_type);
/* Same on an explicit stream. */
int vkflame_dispatch_dequant_async(const void *src, void *dst, uint64_t n_blocks, int quant_type,
                                   void *stream);

/* Fused dequant + linear; replaces the reference's three-dispatch quantised
 * mul_mat chain (shim/hip_runtime_shim.cpp:1102-1172).
 *   W: N rows of K/QK blocks of wtype (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K); ggml layout.
 *   X: M x K activations, xtype VKF_X_F16 (row stride ldx elements) or
 *      VKF_X_Q8_1 (row stride ldx blocks of 36 B; ldx = K/32 when packed).
 *   Y: M x N, ytype VKF_Y_F32 or VKF_Y_F16, row stride ldy elements.
 * Y[m,n] = sum_k X[m,k] * dequant(W)[n,k], fp32 accumulation.  M <= 8 runs
 * the decode GEMV kernel; larger M the tensor-core GEMM. */
int vkflame_quant_linear(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype,
                         int M, int N, int K, int64_t ldx, int64_t ldy, void *stream);

/* vkflame_quant_linear with flags.  VKF_FLAG_STATIC_WEIGHTS: W is not
 * written by the kernel launched just before this call on the same stream
 * (true of model weights), so the kernel may start streaming W while that
 * kernel is still running.  Without the flag all of this call's memory
 * accesses wait for the preceding kernel. */
#define VKF_FLAG_STATIC_WEIGHTS 1u
int vkflame_quant_linear_ex(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype,
                            int M, int N, int K, int64_t ldx, int64_t ldy, unsigned flags, void *stream);

/* ---- column-sharded multi-GPU: decode GEMV fused with the all-gather ----
 * No counterpart in the reference (its runtime is single-device).  The
 * multi-GPU form of the quantised linear: each rank owns a contiguous range
 * of output rows (columns of Y), computes its slice with the decode GEMV and
 * stores it straight into every rank's gathered buffer over NVLink (peer
 * memory mapped with vkflame_ipc_open): no separate collective launch, no
 * fence and no completion signal.
 *
 * Gathered buffer layout (M = 1, fp16): two buffers per rank, `stride` bytes
 * apart; buffer (epoch & 1) holds N / 2 words of 8 bytes, word j =
 * {fp16 Y[2j], fp16 Y[2j + 1], uint32 epoch}.  An aligned 8-byte store is
 * single-copy atomic, so a reader that sees the epoch sees the data.  A call
 * with x_gathered reads X from such a buffer and waits (bounded, inside its
 * kernel) until every word it reads carries its epoch.  epoch is the call
 * site's run count on the device: run t writes words carrying t + 1 and
 * expects t + 1 in the words it reads (every call site runs once per step),
 * and its kernel increments the count when it ends.  Two buffers by parity
 * let a rank run up to one step ahead without overwriting words a slower
 * rank has yet to read, which holds when every step reads at least one
 * gathered X.  One process per GPU; ranks make the same calls in the same
 * order; buffers and counters zeroed on every rank before the first call
 * (host barrier).                                                          */
#define VKF_MAX_RANKS 8
typedef struct vkf_gather {
    int world;                       /* ranks, 1 .. VKF_MAX_RANKS                          */
    int rank;                        /* this rank                                           */
    void *y_rank[VKF_MAX_RANKS];     /* each rank's buffer 0 (mapped here), at this rank's first word */
    int64_t stride;                  /* bytes from a rank's buffer 0 to its buffer 1        */
    int *epoch;                      /* this call site's run count (device int, zero)      */
    int *done;                       /* this rank's CTA counter (device int, zero)          */
    int x_gathered;                  /* X is this rank's buffer 0 of an earlier gather      */
    int64_t x_stride;                /* its bytes from buffer 0 to buffer 1                 */
} vkf_gather_t;

/* Y slice computed by this rank: rows [0, N) of W (this rank's shard),
 * written to every rank's gathered buffers at word offset y_rank.  M = 1,
 * ytype VKF_Y_F16, N even; ldx: X row stride in elements (for a gathered X,
 * the gathered row length); ldy unused (one row). */
int vkflame_quant_linear_gather(const void *W, int wtype, const void *X, int ytype, int M, int N, int K,
                                int64_t ldx, int64_t ldy, unsigned flags, const vkf_gather_t *g, void *stream);

/* ---- a token's decode linears as one persistent kernel (M = 1) ----------
 * No counterpart in the reference.  The linears of one decode step, in
 * order, each computing this rank's shard (rows [0, N) of W) of
 * Y = X dequant(W)^T and storing it into every rank's gathered buffers (the
 * vkf_gather_t word layout above; world size 1: the local buffer) or, at
 * world size 1, into a plain fp16 row.  X is a plain fp16 row (x_src = -1)
 * or the gathered output of an earlier linear of the same chain (x_src = its
 * index; its first K values).  vkflame_chain_run makes ONE cooperative
 * launch (one CTA per SM) that walks every linear: weights stream ahead
 * across linear boundaries while each linear waits (bounded, inside the
 * kernel) for the words of its X.  Formats Q4_K, Q5_K, Q6_K; K a multiple of
 * 256; N even.  One run per step; ranks run the same chain in the same
 * order; the gathered buffers are zeroed on every rank before the first run
 * (host barrier).  The chain owns its run count (epoch) and scratch. */
typedef struct vkf_chain_linear {
    const void *W;                   /* this rank's rows, ggml blocks                        */
    int wtype;                       /* VKF_DEQUANT_Q4_K, Q5_K or Q6_K                        */
    int K, N;                        /* input length; rows of this rank's shard               */
    int x_src;                       /* -1: x_plain; else index of an earlier linear          */
    const void *x_plain;             /* fp16 row of K values, 16-byte aligned                 */
    void *y_rank[VKF_MAX_RANKS];     /* gathered output: each rank's buffer 0, at this rank's first word */
    int64_t y_stride;                /* bytes from a rank's buffer 0 to its buffer 1          */
    void *y_plain;                   /* world size 1 only: plain fp16 output row instead      */
} vkf_chain_linear_t;
typedef struct vkf_chain vkf_chain_t;
#define VKF_CHAIN_TRACE 1u           /* record per-linear timestamps (vkflame_chain_trace)   */
int vkflame_chain_create(const vkf_chain_linear_t *linears, int n, int world, int rank, unsigned flags,
                         vkf_chain_t **chain);
int vkflame_chain_run(vkf_chain_t *chain, void *stream);
/* Run count of the chain's completed runs (synchronous read). */
int vkflame_chain_epoch(const vkf_chain_t *chain, int *epoch);
/* VKF_CHAIN_TRACE: per linear {latest time a CTA had its X ready, latest
 * output store} of the last run, globaltimer ns (host array of 2n). */
int vkflame_chain_trace(const vkf_chain_t *chain, unsigned long long *times);
/* First wait that gave up inside the chain kernel since creation (all zero:
 * none): {role (1 weight producer, 2 reducer, 3 consumer waiting for
 * weights, 4 consumer waiting for a partial slot, 5 activations), linear
 * index, item (or row block / run), CTA}.  Each wait gives up after 2 s. */
int vkflame_chain_status(const vkf_chain_t *chain, int *fail4);
int vkflame_chain_destroy(vkf_chain_t *chain);

/* CUDA IPC for the gathered buffers and counters: a 64-byte handle of the
 * allocation holding dev_ptr plus dev_ptr's byte offset in it; open returns
 * the allocation's base mapped in this process (add the offset). */
int vkflame_ipc_handle(const void *dev_ptr, void *handle64, uint64_t *offset);
int vkflame_ipc_open(const void *handle64, void **base);
int vkflame_ipc_close(void *base);

/* Allocation-free decode GEMV.  No counterpart in the reference: an addition
 * for callers that must not allocate device memory (code inside an
 * allocator callback, processes whose device memory is fully reserved up
 * front, runtimes that forbid allocation after start-up).  Same result as
 * vkflame_quant_linear with xtype VKF_X_F16, but its scratch is a fixed
 * 576 KiB array in this library's device globals (held on every GPU that
 * loads the library until the process exits) instead of per-stream arenas,
 * and it never calls cudaMalloc/cudaFree.
 *   Limits: 1 <= M <= 8, N <= 262144, M * (2K + 160 + K/8) <= 80 KiB,
 *   X rows 16-byte aligned; anything else returns VKF_ERR_INVALID,
 *   VKF_ERR_UNSUPPORTED or VKF_ERR_BADPTR and queues nothing on the stream.
 *   W, X and Y get alignment checks only: their ranges are not validated.
 * A bounded wait that gives up inside its kernel is reported, like every
 * other kernel's, by vkflame_check_kernel_errors (which allocates nothing
 * when only this entry point has run on the device).
 * The first call on a device looks up the scratch's device address
 * (cudaGetSymbolAddress); make that call before any stream capture.
 * Every call shares the one scratch array: calls whose kernels may overlap
 * on the GPU (different streams, or host threads) race and must be
 * serialised by the caller. */
int vkflame_quant_linear_noalloc(const void *W, int wtype, const void *X, void *Y, int ytype, int M, int N,
                                 int K, int64_t ldx, int64_t ldy, void *stream);

/* On-device fp32 -> Q8_1 quantiser (no reference counterpart: the reference
 * only decodes Q8_1, kernels/dequant_q8_1.glsl).  x is M x K fp32 (row stride
 * ldx elements), y receives M rows of K/32 blocks (36 B each), packed.
 * d = max|x|/127 over each 32-value block, q = clamp(round(x/d)) with
 * round-half-away-from-zero, s = d*sum(q); d and s stored as fp16. */
int vkflame_quantize_q8_1(const float *x, void *y, int M, int K, int64_t ldx, void *stream);

/* linear_int8 with per-row and per-channel scales (kernels/linear_int8.glsl,
 * with the defects of the reference's binding corrected):
 *   acc[m,n] = sum_k X[m,k] * W[n,k]            (int32, bit-exact)
 *   Y[m,n]   = fp16(act((acc * sx[m]) * sw[n] + bias[n]))
 * X int8 M x K, W int8 N x K (both K contiguous), sx fp32[M] (NULL = 1),
 * sw fp32[N] (NULL = 1), bias fp16[N] (NULL = none).  If acc_out is not NULL
 * the raw int32 accumulators are also written (M x N). */
int vkflame_linear_int8(const int8_t *X, const int8_t *W, const float *sx, const float *sw,
                        const void *bias, void *Y, int32_t *acc_out, int M, int N, int K,
                        int activation, void *stream);

/* ---- the rest of ggml's kernel-name table (runtime/dispatch.h:60-125) ----
 * fp32 unless stated; pointers are device pointers.  Each restates the
 * reference shader of the same name.  These entry points carry no stream
 * argument (as in the reference): they launch on the calling thread's
 * stream, set with vkflame_set_stream (NULL, the default: the legacy
 * default stream).  vkflame_set_stream has no reference counterpart. */
int vkflame_set_stream(void *stream);
void *vkflame_get_stream(void);   /* the calling thread's stream for these entry points */
/* VKF_EW_* op ids of runtime/dispatch.h:24-38 (kernels/elementwise_f32.glsl). */
#define VKF_EW_SILU 0
#define VKF_EW_GELU_ERF 1
#define VKF_EW_RELU 2
#define VKF_EW_TANH 3
#define VKF_EW_GELU_QUICK 4
#define VKF_EW_NEG 5
#define VKF_EW_SIGMOID 6
#define VKF_EW_SQR 7
#define VKF_EW_SQRT 8
#define VKF_EW_EXP 9
#define VKF_EW_LOG 10
#define VKF_EW_ABS 11
#define VKF_EW_SGN 12
#define VKF_EW_HARDSIGMOID 13
#define VKF_EW_HARDSWISH 14
/* VKF_BINOP_* (runtime/dispatch.h:41-44; kernels/binop_f32.glsl). */
#define VKF_BINOP_ADD 0
#define VKF_BINOP_MUL 1
#define VKF_BINOP_SUB 2
#define VKF_BINOP_DIV 3
/* runtime/dispatch.h:94-98: dst[i] = op(src[i]), i < n (in place allowed). */
int vkflame_dispatch_elementwise_f32(void *ctx, const void *src, void *dst, uint32_t n, uint32_t op);
/* runtime/dispatch.h:107-111: dst[i] = scale * src[i] + bias. */
int vkflame_dispatch_scale_f32(void *ctx, const void *src, void *dst, uint32_t n, float scale, float bias);
/* runtime/dispatch.h:113-117: dst[i] = op(src0[i], src1[i % src1_n]); x / 0 = 0. */
int vkflame_dispatch_binop_f32(void *ctx, const void *src0, const void *src1, void *dst, uint32_t n,
                               uint32_t src1_n, uint32_t op);
/* runtime/dispatch.h:119-123: per row of N, y = x / sqrt(mean(x^2) + eps). */
int vkflame_dispatch_rms_norm_f32(void *ctx, const void *src, void *dst, uint32_t M, uint32_t N, float eps);
/* runtime/dispatch.h:66-69: fp16 X, gamma, Y: y = fp16(x * rrms * gamma). */
int vkflame_dispatch_rms_norm(void *ctx, const void *X, const void *gamma, void *Y, int M, int N, float eps);
/* runtime/dispatch.h:71-74: row softmax, M rows of N. */
int vkflame_dispatch_softmax(void *ctx, const void *X, void *Y, int M, int N);
/* runtime/dispatch.h:100-105: neox RoPE of n_seqs x ne1 rows of ne0 values:
 * value j pairs with j + ne0/2, theta = pos[seq] * theta_scale^j *
 * freq_scale for 2j < n_dims (pass-through beyond).  Every row and pair is
 * computed (the reference's grid, ne1 x n_seqs workgroups for a shader
 * indexed by rows in x and pair groups in y, reached only part of them,
 * runtime/dispatch.cpp:545-548); p0, p1 unused. */
int vkflame_dispatch_rope_neox(void *ctx, const void *src, const void *pos, void *dst, uint32_t ne0, uint32_t ne1,
                               uint32_t n_dims, uint32_t n_seqs, float theta_scale, float freq_scale, uint32_t p0,
                               uint32_t p1);
/* runtime/dispatch.h:81-84: fp16 weight [V x D], int32 indices [B], fp16
 * out [B x D]; an index outside [0, V) gives a zero row. */
int vkflame_dispatch_embedding(void *ctx, const void *weight, const void *indices, void *out, int V, int D, int B);
/* ggml get_rows into fp32 (no reference entry point; the hipLaunchKernel
 * get_rows branch): weight fp32 (weight_f32 = 1) or fp16 [V x D]. */
int vkflame_get_rows(const void *weight, int weight_f32, const void *indices, float *out, int V, int D, int B,
                     void *stream);

/* ---- diagnostics -------------------------------------------------------- */
int vkflame_get_last_error(void);
const char *vkflame_status_string(int status);
/* Synchronises the current device and reports (and clears) the error bits
 * kernels set when a bounded wait gave up: VKF_ERR_TIMEOUT if any was set.
 * Covers every entry point, the allocation-free one included. */
int vkflame_check_kernel_errors(void);
/* Number of kernels this library has launched since load (all devices). */
uint64_t vkflame_kernel_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* VKFLAME_RT_H */
