/*
 * amc.h — C ABI of libamcuda.so, the B200 (sm_100a) realization backend for
 * array-morphisms.
 *
 * The reference library (CHICKEN Scheme, iraikov/array-morphisms) realizes a
 * lazy morphism tree on one host thread by recursive interpretation
 * (realization.scm:92-115).  This library replaces the bodies of that engine:
 * the Scheme host serializes the tree it would have walked into an array of
 * amc_node records (one per morphism node, operands before users) and calls
 * amc_plan_create / amc_plan_execute.  The library composes zero-copy views
 * (realization.scm:649-717), fuses element-wise chains and reductions into
 * single kernels, and launches hand-written sm_100a kernels.  There is no CPU
 * fallback: a node the device path cannot run is an error.
 *
 * Conventions
 *   - Every entry point returns an int status: AMC_OK (0) or an AMC_ERR_* code.
 *     amc_last_error() copies the calling thread's last message.
 *   - Buffers are referred to by 64-bit handles (0 = none).
 *   - Strides and offsets are in ELEMENTS, like the reference's concrete-array
 *     (core.scm:238-247).  A stride may be 0 (broadcast).
 *   - All device work is issued on the current device of the calling thread,
 *     on the stream passed in (NULL = the library's per-device stream).
 */
#ifndef AMC_H
#define AMC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define AMC_OK               0
#define AMC_ERR_INVALID      1   /* bad argument, shape or dtype            */
#define AMC_ERR_UNSUPPORTED  2   /* valid request the device path rejects   */
#define AMC_ERR_CUDA         3   /* CUDA runtime / driver error             */
#define AMC_ERR_OOM          4   /* device allocation failed                */
#define AMC_ERR_STATE        5   /* call out of order (e.g. replay before finalize) */
#define AMC_ERR_INJECTED     6   /* host-side fault injection (AMC_FAULT)   */
#define AMC_ERR_TIMEOUT      7   /* a bounded device wait gave up           */

/* ---------------------------------------------------------------- dtypes
 * Mirrors *supported-dtypes* (core.scm:559-560).  Promotion follows
 * promote-types (core.scm:585-605): f64 > f32 > s64 > s32 > u64 > u32. */
#define AMC_F32 0
#define AMC_F64 1
#define AMC_S32 2
#define AMC_S64 3
#define AMC_U32 4
#define AMC_U64 5

#define AMC_MAX_RANK 8

/* ---------------------------------------------------------------- views
 * A strided window onto a device buffer: the device-side concrete-array
 * (core.scm:238-247: data shape strides offset dtype). */
typedef struct amc_view {
  uint64_t buf;                     /* buffer handle                        */
  int32_t  dtype;                   /* AMC_F32 ...                          */
  int32_t  rank;                    /* 0..AMC_MAX_RANK                      */
  int64_t  shape[AMC_MAX_RANK];
  int64_t  strides[AMC_MAX_RANK];   /* elements                             */
  int64_t  offset;                  /* elements                             */
} amc_view;

/* ---------------------------------------------------------------- element-wise programs
 * The combiner of a compute node (basic-ops.scm:125-133, :258-284, :427-435)
 * as postfix code over a small value stack.  Values carry the reference's
 * numeric tower in two kinds: inexact (IEEE double) and exact (int64).
 * Loads of f32/f64 operands push inexact values, integer operands push exact
 * values; arithmetic on two exact values stays exact except DIV, which
 * yields inexact (the reference yields a rational that only survives until
 * the node's store truncates it).  The result of a node program is stored
 * with the reference's typed-vector-set! conversion (core.scm:649-658). */
typedef struct amc_insn {
  int32_t op;      /* AMC_OP_* */
  int32_t a;       /* operand index for LOAD, dtype for CVT                 */
  double  imm;     /* constant for CONST / ICONST                           */
} amc_insn;

#define AMC_OP_LOAD     1   /* push operand a                                */
#define AMC_OP_CONST    2   /* push inexact imm                              */
#define AMC_OP_ICONST   3   /* push exact (int64)imm                         */
#define AMC_OP_CVT      4   /* round top of stack as a store to dtype a      */
/* unary */
#define AMC_OP_NEG     10
#define AMC_OP_ABS     11
#define AMC_OP_FLOOR   12
#define AMC_OP_CEIL    13
#define AMC_OP_SQRT    14
#define AMC_OP_EXP     15
#define AMC_OP_LOG     16
#define AMC_OP_SIN     17
#define AMC_OP_COS     18
#define AMC_OP_TAN     19
#define AMC_OP_RELU    20   /* (max 0.0 (exact->inexact x))                  */
#define AMC_OP_SIGMOID 21   /* 1/(1+exp(-x))                                 */
#define AMC_OP_TANH    22   /* (e2-1)/(e2+1), e2 = exp(2x), basic-ops.scm:279-282 */
/* binary (pops b then a, pushes a op b) */
#define AMC_OP_ADD     40
#define AMC_OP_SUB     41
#define AMC_OP_MUL     42
#define AMC_OP_DIV     43
#define AMC_OP_POW     44
#define AMC_OP_MAX     45
#define AMC_OP_MIN     46
#define AMC_OP_GT      50   /* comparisons push inexact 1.0 / 0.0            */
#define AMC_OP_LT      51
#define AMC_OP_EQ      52
#define AMC_OP_GE      53
#define AMC_OP_LE      54

#define AMC_PROG_MAX   64   /* instructions per fused program                */
#define AMC_STACK_MAX  16

/* ---------------------------------------------------------------- reduction ops
 * morph-reduce (basic-ops.scm:522-608); output dtype by
 * infer-reduction-dtype (core.scm:607-621). */
#define AMC_RED_SUM  0
#define AMC_RED_MEAN 1
#define AMC_RED_PROD 2
#define AMC_RED_MAX  3
#define AMC_RED_MIN  4

/* ---------------------------------------------------------------- pad modes (structural-ops.scm:449-507) */
#define AMC_PAD_CONSTANT 0
#define AMC_PAD_EDGE     1
#define AMC_PAD_REFLECT  2

/* ---------------------------------------------------------------- plan nodes
 * One record per morphism node of the tree the reference's realize walks.
 * Operands are earlier records (in[] < own index).  The last record is the
 * root.  Kind-specific parameters:
 *   LEAF       leaf = device view of a concrete-array
 *   RESHAPE    shape = target shape                  (structural-ops.scm:49-137)
 *   TRANSPOSE  iparam[0..rank) = permutation         (:167-226)
 *   SLICE      iparam[0..r) = starts, iparam[8..8+r) = steps (:245-335)
 *   MAP        prog/prog_len over n_in operands, numpy broadcasting (basic-ops.scm:40-123, :475-507)
 *   REDUCE     iparam[0] = AMC_RED_*, iparam[1] = axis bit mask, iparam[2] = keepdims (basic-ops.scm:522-608)
 *   PAD        iparam[0] = mode, iparam[1+2i], iparam[2+2i] = before/after of axis i; fparam[0] = value
 *   IM2COL     iparam[0..6) = KH KW SH SW PH PW      (structural-ops.scm:513-627)
 *   COL2IM     iparam[0..6) = KH KW SH SW PH PW      (structural-ops.scm:629-727)
 *   STACK      iparam[0] = axis, operands via in_ext (structural-ops.scm:729-790)
 *   CONCAT     iparam[0] = axis, operands via in_ext
 *   MATMUL     2 operands (M,K)x(K,N)                (blas-exec.scm:227-260)
 *   MATVEC     2 operands (M,N)x(N)
 *   DOT        2 operands (N)x(N) -> ()
 *   ATTENTION  3 operands Q K V, fparam[0] = scale   (blas-exec.scm:334-398)
 *   SCAN       2 operands init (element shape E) and x (n, E...), prog over LOAD 0 = the
 *              accumulator and LOAD 1 = element i; iparam[0] = 1 keeps every accumulator
 *              (batch-scan, result (n, E...)), 0 the last (batch-fold, result E); the
 *              accumulator is rounded to the init dtype after each step, as the per-element
 *              tree of batch-ops.scm:278-322 stores it.  Replaces that tree of n map nodes.
 *   OUTPUTS    the last node only: its operands are the roots of one program realized
 *              together, every shared node once (the outputs of ssa-realize, ssa.scm:1130-1156
 *              and :1661-1749); amc_plan_result_at gives each.
 * The planner recognises reshape(matmul(W, im2col(X))) on one f32 (C, H, W)
 * image as a convolution (detect-conv2d-pattern, realization.scm:136-164) and
 * runs amc_conv2d_fwd_f32 on it; an ATTENTION node of contiguous f32 operands
 * with head dim 64 and n a multiple of 128 runs the tensor-core kernel. */
#define AMC_N_LEAF      1
#define AMC_N_RESHAPE   2
#define AMC_N_TRANSPOSE 3
#define AMC_N_SLICE     4
#define AMC_N_MAP       5
#define AMC_N_REDUCE    6
#define AMC_N_PAD       7
#define AMC_N_IM2COL    8
#define AMC_N_COL2IM    9
#define AMC_N_STACK    10
#define AMC_N_CONCAT   11
#define AMC_N_MATMUL   12
#define AMC_N_MATVEC   13
#define AMC_N_DOT      14
#define AMC_N_ATTENTION 15
#define AMC_N_SCAN     16
#define AMC_N_OUTPUTS  17

#define AMC_NODE_MAX_IN 4

typedef struct amc_node {
  int32_t  kind;
  int32_t  dtype;                   /* result dtype                          */
  int32_t  rank;                    /* result rank                           */
  int32_t  n_in;                    /* operand count                         */
  int64_t  shape[AMC_MAX_RANK];     /* result shape                          */
  int32_t  in[AMC_NODE_MAX_IN];     /* operand record indices (n_in <= 4)    */
  const int32_t* in_ext;            /* operand indices when n_in > 4         */
  int64_t  iparam[24];
  double   fparam[4];
  const amc_insn* prog;             /* MAP program                           */
  int32_t  prog_len;
  int32_t  _pad;
  amc_view leaf;                    /* LEAF view                             */
} amc_node;

/* ---------------------------------------------------------------- runtime */
int amc_last_error(char* buf, size_t len);
int amc_version(int* major, int* minor);
int amc_device_count(int* n);
int amc_init(int device);           /* make device current, create its stream */
int amc_shutdown(void);             /* free every buffer, plan and arena      */
int amc_synchronize(void);          /* wait for the current device's stream   */

/* ---------------------------------------------------------------- buffers
 * Device storage for SRFI-4 vectors (core.scm:627-658). */
int amc_buf_create(int32_t dtype, int64_t nelem, uint64_t* out);
int amc_buf_wrap(void* devptr, int32_t dtype, int64_t nelem, uint64_t* out);  /* not owned */
int amc_buf_upload(uint64_t h, const void* host, int64_t bytes, int64_t byte_offset);
int amc_buf_download(uint64_t h, void* host, int64_t bytes, int64_t byte_offset);
int amc_buf_upload_async(uint64_t h, const void* host, int64_t bytes, int64_t byte_offset, void* stream);
int amc_buf_download_async(uint64_t h, void* host, int64_t bytes, int64_t byte_offset, void* stream);
/* Device-to-device copy between buffers, stream-ordered (the in-place
 * update of a vector, e.g. a parameter after an optimizer step,
 * f64vector-set! over a whole vector; core.scm:649-658). */
int amc_buf_copy_async(uint64_t dst, int64_t dst_byte_offset, uint64_t src, int64_t src_byte_offset, int64_t bytes,
                       void* stream);
int amc_buf_devptr(uint64_t h, void** out);
int amc_buf_info(uint64_t h, int32_t* dtype, int64_t* nelem);
int amc_buf_free(uint64_t h);

/* ---------------------------------------------------------------- realize
 * amc_plan_create lowers one serialized tree; amc_plan_execute runs it.
 * Replaces realize / realize-morphism-expr / realize-reduction
 * (realization.scm:92-115, :398-468, :1274-1307). */
int amc_plan_create(const amc_node* nodes, int32_t n, uint64_t* plan);
int amc_plan_execute(uint64_t plan, void* stream);
/* The root's result: a view of a plan-owned (or context-owned) buffer, or of
 * a leaf buffer when the root is a zero-copy view (realization.scm:649-717). */
int amc_plan_result(uint64_t plan, amc_view* out);
/* The results of a plan whose last node is OUTPUTS (one per operand, in
 * order; a single-root plan has one).  The caller owns one reference. */
int amc_plan_result_count(uint64_t plan, int32_t* n);
int amc_plan_result_at(uint64_t plan, int32_t i, amc_view* out);
/* Number of kernel launches one execute issues, and allocations it made. */
int amc_plan_stats(uint64_t plan, int32_t* launches, int32_t* buffers, int64_t* bytes);
/* Capture the plan's launches into a CUDA graph; later executes replay it. */
int amc_plan_capture_graph(uint64_t plan, void* stream);
int amc_plan_destroy(uint64_t plan);

/* ---------------------------------------------------------------- context
 * realize/ctx (context.scm:17-39, :125-161): plans created against a context
 * in trace mode allocate and record every intermediate buffer; after
 * amc_ctx_finalize the records are coloured greedily by birth order
 * (context.scm:325-412) into ONE device arena, and plans created in replay
 * mode bind their buffers to arena offsets: replay performs no allocation. */
int amc_ctx_create(uint64_t* ctx);
int amc_plan_create_ctx(uint64_t ctx, const amc_node* nodes, int32_t n, uint64_t* plan);
int amc_ctx_pin_output(uint64_t ctx, uint64_t plan);       /* context.scm:190-200 */
int amc_ctx_finalize(uint64_t ctx);                         /* context.scm:133-154 */
int amc_ctx_reset(uint64_t ctx);                            /* context.scm:156-161 */
/* Run again a plan created in this context's replay mode, on its arena
 * buffers, without re-planning (execute-replay-plan, ssa.scm:1519-1654).  The
 * context counter must be at the plan's first allocation (after
 * amc_ctx_reset, or after the plans created before it), and moves past the
 * plan's allocations. */
int amc_ctx_replay(uint64_t ctx, uint64_t plan, void* stream);
/* stats: allocations recorded, buffers after colouring, arena bytes, mode (0 trace, 1 replay) */
int amc_ctx_stats(uint64_t ctx, int32_t* allocations, int32_t* buffers, int64_t* arena_bytes, int32_t* mode);
int amc_ctx_destroy(uint64_t ctx);
/* The greedy colouring itself on caller-supplied records (for tests and for
 * hosts that keep their own trace): sizes in elements, last_use per record
 * after lifetime extension is computed here from inputs (context.scm:282-295).
 * inputs: flat array, record i owns inputs[in_off[i] .. in_off[i+1]).
 * assignment[i] receives the buffer id; n_buffers the count. */
int amc_colour(int32_t n, const int32_t* dtypes, const int64_t* sizes,
               const int32_t* in_off, const int32_t* inputs, const int32_t* pinned,
               int32_t* assignment, int32_t* n_buffers);

/* ---------------------------------------------------------------- BLAS backend record
 * Normalized kernel interface of make-blas-backend (blas-exec.scm:16-46,
 * :137-148; adapter pattern chicken-blas-backend.scm:49-151).  Host pointers,
 * row-major, contiguous; C is updated in place.  Each call stages operands
 * through device memory and returns after the result is back on the host. */
int amc_blas_dgemm(int32_t M, int32_t N, int32_t K, double alpha, const double* A, const double* B, double beta, double* C);
int amc_blas_sgemm(int32_t M, int32_t N, int32_t K, float alpha, const float* A, const float* B, float beta, float* C);
int amc_blas_dgemm_strided(int32_t M, int32_t N, int32_t K, double alpha, const double* A, int32_t lda, int32_t transA,
                           const double* B, int32_t ldb, int32_t transB, double beta, double* C);
int amc_blas_sgemm_strided(int32_t M, int32_t N, int32_t K, float alpha, const float* A, int32_t lda, int32_t transA,
                           const float* B, int32_t ldb, int32_t transB, float beta, float* C);
int amc_blas_dgemv(int32_t M, int32_t N, double alpha, const double* A, const double* x, double beta, double* y);
int amc_blas_sgemv(int32_t M, int32_t N, float alpha, const float* A, const float* x, float beta, float* y);
int amc_blas_ddot(int32_t N, const double* x, const double* y, double* out);
int amc_blas_sdot(int32_t N, const float* x, const float* y, float* out);
int amc_blas_daxpy(int32_t N, double alpha, const double* x, double* y);
int amc_blas_saxpy(int32_t N, float alpha, const float* x, float* y);

/* ---------------------------------------------------------------- fused workloads on device views
 * Entry points for the hot paths the planner also reaches, callable directly
 * on device buffers (no staging) for hosts that already hold device data.
 *
 * Windowed FIR / polyphase filter bank (example-08 domain; the tree
 * morph-reduce 'sum (morph* (transpose (reshape (im2col x (1 KW) (1 S)))) h) over taps):
 *   out[b, f, m] = sum_{t<T} h[t*M + m] * x[b*xs + f*S + t*M + m]
 * f32, accumulated in tap order with the reference's per-node rounding. */
int amc_window_fir_f32(const float* x, int64_t batch, int64_t x_batch_stride, int64_t frames,
                       int64_t hop, int32_t taps, int32_t branches, const float* h,
                       float* out, void* stream);

/* Linear regression by gradient descent with the loss mean((X w - y)^2)
 * (example-09 / ssa.scm replay of the MSE step).  One launch sequence per
 * step: a fused pass over X producing per-block partial gradients and loss,
 * a fixed-order reduction, and the update w -= lr * grad.  X (rows, d) and
 * y (rows) are this device's rows of a problem with n_total rows; the
 * gradient of each row is dr = g*r + g*r with g = 1/n_total (the mean rule).
 * grad_loss holds d gradient sums followed by the sum of squared residuals;
 * hosts sharding rows across devices sum grad_loss over devices (in a fixed
 * order) between amc_linreg_reduce and amc_linreg_update.
 * amc_linreg_step runs the three launches on one device; partials must hold
 * amc_linreg_partials_count(rows, d) * (d + 1) doubles. */
int amc_linreg_partials_count(int64_t rows, int32_t d, int32_t* n_partials);
int amc_linreg_partials(const double* X, const double* y, const double* w, int64_t rows, int32_t d, int64_t n_total,
                        double* partials, void* stream);
int amc_linreg_reduce(const double* partials, int32_t n_partials, int32_t d, double* grad_loss, void* stream);
int amc_linreg_update(double* w, const double* grad_loss_sum, int32_t d, int64_t n_total, double lr,
                      double* loss_out, void* stream);
int amc_linreg_step(const double* X, const double* y, double* w, int64_t rows, int32_t d, double lr,
                    double* partials, double* grad_loss, double* loss_out, void* stream);

/* Linear-regression step that allocates nothing.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory —
 * hosts whose device memory belongs to another allocator (a framework's
 * caching allocator, a fixed per-process budget) or that must not call
 * cudaMalloc, which can synchronise the device, inside a timed loop.
 * Same arithmetic as amc_linreg_step, but the partial sums live in a static
 * device array of 262144 doubles (2 MiB, held by every GPU that loads the
 * library until exit); calls needing more, (partials + 1) * (d + 1) doubles
 * with partials = amc_linreg_partials_count(rows, d), are rejected with
 * AMC_ERR_INVALID.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture.  Every call shares the one array and every
 * scratch entry is written before it is read; calls that overlap on the GPU
 * (different streams, or different host threads on one device) race.
 * Pass a stream, or call amc_init first, so no library stream is created here. */
int amc_linreg_step_noalloc(const double* X, const double* y, double* w, int64_t rows, int32_t d, double lr,
                            double* loss_out, void* stream);

/* Scaled dot-product attention, streaming softmax (realization.scm:279-396):
 * Q (B, n, dk), K (B, n, dk), V (B, n, dv) row-major contiguous per block;
 * lse (B, n) receives the natural-log row log-sum-exp (may be NULL in the
 * forward).  With dk = dv = 64, n a multiple of 128 and 16-byte-aligned
 * pointers both directions run on the tcgen05 tensor cores with operands
 * rounded to tf32 (within 2e-3 of the output scale); other shapes run f32
 * SIMT kernels.  The backward uses no atomics: repeated calls give identical
 * bits.  The reference has no attention gradient; the backward is the
 * standard softmax-attention VJP.  Per-device scratch is allocated on first
 * use and kept. */
int amc_attention_fwd_f32(const float* Q, const float* K, const float* V, float* O, float* lse,
                          int64_t blocks, int32_t n, int32_t dk, int32_t dv, float scale, void* stream);
int amc_attention_bwd_f32(const float* Q, const float* K, const float* V, const float* O, const float* dO,
                          const float* lse, float* dQ, float* dK, float* dV,
                          int64_t blocks, int32_t n, int32_t dk, int32_t dv, float scale, void* stream);

/* 2-D convolution, NCHW, stride/pad, as the reference's im2col + GEMM
 * (realization.scm:166-252) and its adjoints via col2im (realization.scm:1196-1268).
 * C = K = 64, 3x3, stride 1, pad 1 (forward/data gradient: W <= 62, W % 4 == 0,
 * H even; weight gradient: W % 4 == 0, H*W % 32 == 0) run as tcgen05 implicit
 * GEMMs with operands rounded to tf32 (within 2e-3 of the output scale); other
 * shapes run direct kernels with double accumulation (the reference's values).
 * The weight gradient's split-K partials are summed in a fixed order. */
int amc_conv2d_fwd_f32(const float* X, const float* W, float* Y, int32_t N, int32_t C, int32_t H, int32_t Wd,
                       int32_t K, int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW, void* stream);
int amc_conv2d_dgrad_f32(const float* dY, const float* W, float* dX, int32_t N, int32_t C, int32_t H, int32_t Wd,
                         int32_t K, int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW, void* stream);
int amc_conv2d_wgrad_f32(const float* X, const float* dY, float* dW, int32_t N, int32_t C, int32_t H, int32_t Wd,
                         int32_t K, int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW, void* stream);

/* ---------------------------------------------------------------- multi-GPU
 * Fixed-order sum over the GPUs of one node (one process per GPU), the
 * reduction that crosses the batch axis of a sharded workload
 * (batch-ops.scm:241-254 folds per-element results in index order).  Each
 * rank creates a group (one device allocation exported by CUDA IPC; its
 * 64-byte handle is written to handle_out), the host exchanges the handles
 * (e.g. an all-gather), and every rank opens the group with all `world`
 * handles in rank order.  amc_peer_sum then replaces out[i] by
 * sum over ranks q = 0 .. world-1 of rank q's src[i], added in that order in
 * double: every rank calls it with the same n and dtype in the same order.
 * Each rank pushes its vector into every rank's memory over NVLink and waits
 * (bounded; AMC_ERR_TIMEOUT at amc_synchronize when a rank never arrives)
 * for the others.  Destroy only after every rank finished its last sum (a
 * host barrier). */
int amc_peer_group_create(int32_t rank, int32_t world, int64_t max_elems, uint64_t* group, void* handle_out);
int amc_peer_group_open(uint64_t group, const void* handles);
int amc_peer_sum(uint64_t group, const void* src, int64_t n, int32_t dtype, void* out, void* stream);
int amc_peer_group_destroy(uint64_t group);

/* Tensor-core throughput probe (diagnostic; no reference counterpart): one
 * CTA per SM, `warps` (1..4) threads each issue iters x 4 back-to-back
 * tcgen05.mma kind::tf32 products of M=128, N=n (32, 64, 128 or 256), K=8
 * into their own accumulator.  B is read from shared memory; A from shared
 * memory (a_tmem = 0) or from tensor memory (a_tmem = 1).  *tflops receives
 * the rate reached.  n=256 with one warp and a_tmem = 0 gives the dense TF32
 * peak, the roofline denominator of the tensor-core kernels.  Synchronizes
 * the stream. */
int amc_tc_peak_tf32(int32_t n, int32_t warps, int32_t a_tmem, int32_t iters, double* tflops, void* stream);

/* Bounded-wait probe (diagnostic; no reference counterpart): runs the bounded
 * mbarrier wait of the TMA/tensor-core kernels alone on a tiny launch.  The
 * barrier expects one arrival, which the kernel makes only when arrive = 1;
 * the wait polls at most `limit` (1..2^22) times.  Returns AMC_OK when the
 * barrier completed and AMC_ERR_TIMEOUT when the wait ran out, after the
 * kernel recorded the timeout and returned (the context stays usable).
 * Synchronizes the stream. */
int amc_probe_bounded_wait(int32_t limit, int32_t arrive, void* stream);

/* Launch counter (diagnostic; no reference counterpart): how many column-fold
 * reductions (adjacent outputs, closed-form element program, TMA tiles) this
 * process has launched, so tests can tell that path from the staged one. */
int amc_colfold_launch_count(int64_t* count);

#ifdef __cplusplus
}
#endif
#endif /* AMC_H */
