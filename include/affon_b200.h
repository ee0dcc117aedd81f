/*
 * affon_b200 — C ABI of the sm_100a kernel library for Affon's affine
 * group-quantized matmul (`affon:ops.quantized_matmul`).
 *
 * This is the boundary the reference's CUDA device backend would bind.  In the
 * reference the operation reaches its backend through
 *   src/js/ops.ts:69-79 (public op) -> src/js/compute/program.ts:481-495
 *   (validation, f32 [M,N] result spec) -> src/js/compute/native.zig:731-746,851
 *   (lowering to compute.OpTag.quantized_matmul with {bits, group_size}) ->
 *   the compute core's physical selection of `cuda_quantized_matmul`
 *   (docs/core/quantized-inference.md:175-181) -> the CUDA backend launch.
 * The only in-tree C-ABI form of the operation is the Cyna adapter
 * `compute_core_run_quantized_matmul_f32` (src/support/compute_core_cyna.zig:29-45);
 * its status codes (0 ok, 1 invalid shape) and its rule that the output is left
 * untouched on error are kept here.
 *
 * Plain pointers and sizes only.  Device pointers are caller-owned; the
 * library never allocates outputs.  Launches are asynchronous on the stream of
 * the context; validation happens on the host before any launch.
 */
#ifndef AFFON_B200_H
#define AFFON_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AFFON_B200_ABI_VERSION 1

/* Status codes.  0/1 follow compute_core_cyna.zig:1000-1032 (0 ok,
 * 1 InvalidShape); the rest name the reference's other failure classes. */
typedef enum affon_b200_status {
    AFFON_B200_OK = 0,
    AFFON_B200_INVALID_SHAPE = 1,   /* program.ts:484-493 shape/option rules */
    AFFON_B200_UNSUPPORTED = 2,     /* `unsupported_lowering` (docs/core/backend-support.md:73-75) */
    AFFON_B200_CUDA_ERROR = 3,      /* a CUDA runtime call failed */
    AFFON_B200_TIMEOUT = 4,         /* a bounded wait gave up (tensor-parallel path) */
    AFFON_B200_GUARD_MISMATCH = 5,  /* denseInputs guard (docs/core/optimization-and-profiling.md:143-151) */
    AFFON_B200_POLICY_REJECTED = 6, /* numericalPolicy rejects the candidate's class (quantized-inference.md:175-177) */
    AFFON_B200_INVALID_ARG = 7,     /* null pointer, unknown enum, bad context */
    AFFON_B200_INVALID_DTYPE = 8    /* program.ts:487 dtype rule */
} affon_b200_status;

typedef enum affon_b200_dtype {
    AFFON_B200_F32 = 0,
    AFFON_B200_BF16 = 1,
    AFFON_B200_U32 = 2,
    AFFON_B200_U64 = 3  /* tensor-parallel max-reduction of packed argmax keys */
} affon_b200_dtype;

/* CompileOptions.numericalPolicy (docs/core/optimization-and-profiling.md:124-130). */
typedef enum affon_b200_policy {
    AFFON_B200_POLICY_BACKEND_EQUIVALENT = 0, /* default: accepts `reassociated` */
    AFFON_B200_POLICY_EXACT_ONLY = 1,         /* rejects every quantized candidate */
    AFFON_B200_POLICY_APPROXIMATE = 2         /* also accepts bf16-rounded weights */
} affon_b200_policy;

/* Numerical class of a physical implementation. */
typedef enum affon_b200_numerics {
    AFFON_B200_EXACT = 0,
    AFFON_B200_REASSOCIATED = 1,
    AFFON_B200_APPROXIMATE = 2
} affon_b200_numerics;

/* A logical rank-two view: shape, element strides and a byte offset from the
 * base pointer (quantized-inference.md:51-52: "logical indices are mapped
 * through their element strides and byte offsets"). */
typedef struct affon_b200_view {
    int64_t rows;
    int64_t cols;
    int64_t row_stride;  /* elements */
    int64_t col_stride;  /* elements */
    int64_t byte_offset; /* bytes from the base pointer */
} affon_b200_view;

/* One quantized_matmul node: y[M,N] = x[M,K] . decode(w)[N,K]^T with
 * decode(w)[n,k] = s[n,k/g] * q[n,k] + b[n,k/g] (quantized-inference.md:59-61).
 * x: [M,K] f32|bf16; w: [N,K*bits/32] u32; s, b: [N,K/g] f32|bf16 (same dtype);
 * y: [M,N] f32 (the reference result dtype, program.ts:494) or bf16
 * (an extension for decoder use; selecting it opts into bf16 rounding). */
typedef struct affon_b200_qmm_desc {
    uint32_t struct_size;     /* sizeof(affon_b200_qmm_desc) */
    int32_t bits;             /* 2, 4 or 8 */
    int64_t group_size;       /* positive */
    int32_t x_dtype;          /* affon_b200_dtype */
    int32_t param_dtype;      /* dtype of scales and biases */
    int32_t y_dtype;          /* AFFON_B200_F32 (default) or AFFON_B200_BF16 */
    int32_t numerical_policy; /* affon_b200_policy */
    int32_t dense_inputs;     /* nonzero: every input must be dense with zero offset */
    int32_t reserved;
    affon_b200_view x, w, s, b, y;
} affon_b200_qmm_desc;

/* Result of physical selection (the compute core's `implementation_id`,
 * docs/core/optimization-and-profiling.md:369-380). */
typedef struct affon_b200_selection {
    char implementation_id[64]; /* e.g. "cuda_quantized_matmul.sm100_qmv_b4_g64" */
    int32_t implementation_version;
    int32_t numerical_class;    /* affon_b200_numerics */
    int32_t splits;             /* K segments combined per output tile, at most (1 = none) */
    int32_t reserved;
    char reason[256];
} affon_b200_selection;

typedef struct affon_b200_ctx affon_b200_ctx;

/* Library / device identification. */
int affon_b200_abi_version(void);
/* Message of the last failing call on this thread ("" if none). */
const char *affon_b200_last_error(void);

/* Context: one per (device, stream).  device_ordinal < 0 reads
 * AFFON_CUDA_DEVICE (docs/runtime/configuration.md:19,99-104; default 0).
 * cuda_stream is a cudaStream_t (NULL = legacy default stream).  The context
 * owns a split-K workspace; calls on one context must not overlap on the GPU
 * from different streams. */
int affon_b200_ctx_create(int device_ordinal, void *cuda_stream, affon_b200_ctx **out);
int affon_b200_ctx_destroy(affon_b200_ctx *ctx);
int affon_b200_ctx_set_stream(affon_b200_ctx *ctx, void *cuda_stream);
int affon_b200_ctx_device(const affon_b200_ctx *ctx);
/* Overlap mode (default off): launch the decode kernels (qmv, its prologue,
 * decode attention, embed, finalize) with programmatic dependent launch, so
 * each may start while the kernel before it in the stream finishes and
 * prefetch its weights, scales and biases -- never its activations -- before
 * waiting for that kernel.  Enable it only when no kernel launched directly
 * before one of these writes its weights, scales or biases. */
int affon_b200_ctx_set_overlap(affon_b200_ctx *ctx, int enable);

/* Test hook of the decode qmv's split-K combine, process-wide: the limit of
 * its bounded wait for the other contributors of a block (0 = the default
 * 4 s) and arrivals it waits for beyond the real contributors (0 in normal
 * use; 1 makes every shared block's wait run out, so a test can check that
 * the timeout is reported and the next launch is correct). */
int affon_b200_debug_set_combine_wait(uint64_t limit_ns, uint32_t extra_arrivals);

/* Test hook of the reassociated prefill qmm, process-wide: the most
 * activation rows one launch pass takes (rounded down to whole 256-row tiles;
 * 0 = as many as the workspace holds).  Large M is always processed in row
 * slices whose group sums fit the workspace; a small cap lets a test run
 * several slices on a small problem. */
int affon_b200_debug_set_slice_rows(int64_t rows);

/* Grow the workspace to at least `bytes` (allocates; never called implicitly
 * by a launch, so launches can be captured in CUDA graphs). */
int affon_b200_ctx_reserve_workspace(affon_b200_ctx *ctx, size_t bytes);

/* Wait for the context's stream and report device-side failures since the
 * last check (and clear them): AFFON_B200_TIMEOUT when a kernel's bounded wait
 * gave up, AFFON_B200_INVALID_ARG when a kernel found a device-resident
 * position or token out of range. */
int affon_b200_ctx_synchronize(affon_b200_ctx *ctx);

/* Validation alone (program.ts:481-495 plus the descriptor's own checks). */
int affon_b200_validate(const affon_b200_qmm_desc *desc);

/* Physical selection without launching.  Replaces the compute core's
 * candidate discovery -> numerical-policy filter -> implementation choice
 * for quantized_matmul (quantized-inference.md:132-140,175-181). */
int affon_b200_select(const affon_b200_qmm_desc *desc, affon_b200_selection *out);

/* Launch quantized_matmul on the context's stream.  All pointers are device
 * pointers (base of each view).  y is untouched when the call fails before
 * the launch.  Replaces the reference's `cuda_quantized_matmul` backend
 * kernel (quantized-inference.md:177-181). */
int affon_b200_qmm(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                   const void *s, const void *b, void *y);

/* Same with the selection the launch used reported in `sel` (may be NULL). */
int affon_b200_qmm_explain(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                           const void *s, const void *b, void *y, affon_b200_selection *sel);

/* Host-buffer form: copies the four inputs host->device, launches, copies y
 * device->host and synchronises the context stream.  Staging buffers are
 * owned by the context and reused across calls.  This is the synchronous
 * caller-owned-host-buffer contract of compute_core_cyna.zig:1000-1032. */
int affon_b200_qmm_host(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                        const void *s, const void *b, void *y);

/* The reference's C-ABI shape (compute_core_cyna.zig:29-45) on the GPU:
 * dense f32 activations / parameters / output, host buffers, element counts,
 * synchronous.  Status 0 ok, 1 invalid shape (output untouched), other =
 * core failure.  Uses a per-thread default context on AFFON_CUDA_DEVICE. */
int affon_b200_compute_core_run_quantized_matmul_f32(
    const float *activation, size_t activation_count, const uint32_t *weights, size_t weight_count,
    const float *scales, size_t scale_count, const float *biases, size_t bias_count, float *output,
    size_t output_count, size_t rows, size_t depth, size_t columns, size_t bits, size_t group_size);

/* Decode qmv without any device allocation.  (No counterpart in the
 * reference: an addition for callers that cannot let a library allocate
 * device memory -- runtimes that own all GPU memory in a pre-reserved arena,
 * or plugin hosts whose allocator is the only one allowed to call the
 * driver.)  Same contract and results as affon_b200_qmm for the decode qmv
 * (M <= 32, 4/8-bit, group 64, bf16 activations and parameters); other
 * descriptors return AFFON_B200_UNSUPPORTED.  No context is needed: the launch
 * goes to `cuda_stream` on the current device, and the kernel's scratch lives
 * in a static 8 MiB device array that every GPU loading this library holds
 * until exit; shapes whose partial sums exceed it (large M*N) are rejected
 * with AFFON_B200_UNSUPPORTED and a message.  The first call on a device looks
 * up that array's device address, so make it before any stream capture.  All
 * calls share the one array and each clears what must start at zero: calls
 * that overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller. */
int affon_b200_qmv_noalloc(const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w, const void *s,
                           const void *b, void *y, void *cuda_stream);

/* Status of the last affon_b200_qmv_noalloc launch on the current device:
 * synchronises `cuda_stream`, reads the static array's status word into
 * *status_out (0 = fine) and returns AFFON_B200_TIMEOUT when a bounded wait of
 * that launch gave up (its output is then invalid).  Read it before the next
 * call, which clears the word.  Allocates nothing. */
int affon_b200_qmv_noalloc_status(void *cuda_stream, uint32_t *status_out);

/* ---------------------------------------------------------------------------
 * Decoder building blocks.  No counterpart in the reference, which has no
 * quantized decoder (packages/@affon/models/src/llama/model.ts:64-78 uses
 * dense matmuls); they run the BASELINE Llama-shaped decode around the
 * quantized linears, with the decoder's norms, residual adds, gated
 * activation and argmax fused into the qmv. */

/* Activations in the decode qmv's order.  For 4-bit codes the decode qmv
 * reads x in "pair order": within every 8 consecutive columns,
 * [x0 x4 x1 x5 x2 x6 x3 x7] (8-bit codes: natural order).  mode 0: src is
 * bf16 [rows][ld_src]; mode 1: src is an f32 residual stream h and the output
 * is bf16(h[m][k] * rsqrt(sum_k h[m][k]^2 / cols + eps) * gamma[k]), the sum
 * taken from ss ([ss_tiles][32] f32 partial sums, summed in a fixed order).
 * rows <= 32; dst is bf16 [rows][ld_dst]. */
int affon_b200_qmv_prep(affon_b200_ctx *ctx, int mode, const void *src, int64_t ld_src, const float *ss,
                        int ss_tiles, const void *gamma, float eps, int rows, int cols, int bits, void *dst,
                        int64_t ld_dst);

/* Fusions of the decode qmv.  x_mode 0: x is natural-order bf16 (the call
 * converts it); x_mode 1: x is already in the qmv's order (affon_b200_qmv_prep
 * or a fused producer wrote it).  epilogue 0: store y; epilogue 1:
 * h_out[m][n] += y[m][n] (f32) and ss_out[n/16][m] (rows of 32 floats) = sum
 * of the squares of the 16 updated h_out entries; epilogue 2: for n%16 < 8 (weight tiles of 8 gate
 * rows then the 8 matching up rows), act[m][8*(n/16) + n%8] =
 * bf16(silu(y[m][n]) * y[m][n+8]), in pair order within each 8 columns when
 * act_pair_order is set; epilogue 3: atomicMax(amax[m], key(y[m][n]) << 32 |
 * (0xffffffff - n)) with an order-preserving key (lowest index wins ties;
 * amax must start at 0). */
typedef struct affon_b200_qmv_fusion {
    uint32_t struct_size;
    int32_t x_mode;
    int32_t epilogue;
    int32_t act_pair_order;
    float *h_out;
    int64_t ld_h_out;
    float *ss_out;
    void *act;
    int64_t ld_act;
    unsigned long long *amax;
    int64_t index_offset; /* epilogue 3: added to n in the key (the first row of a vocabulary shard) */
    /* Row-scale mode (row_ss != NULL): x holds bf16(h * gamma), the
     * activations before RMSNorm's row scale, and every output of row m is
     * multiplied by rsqrt(sum_k h[m][k]^2 / K + eps) -- the fused RMSNorm --
     * with the sums of squares from row_ss ([ss_tiles][32] partial sums). */
    const float *row_ss;
    int32_t ss_tiles;
    float eps;
    /* Epilogue 1 extra output (next_x != NULL): next_x[m][c(n)] =
     * bf16(h_out[m][n] * next_gamma[n]) after the residual update, c(n) in
     * the 4-bit pair order when next_pair_order -- the next projection's
     * row-scale-mode activations. */
    const void *next_gamma;
    void *next_x;
    int64_t ld_next_x;
    int32_t next_pair_order;
    /* Epilogue 4 (tensor parallel, after affon_b200_tp_exchange_reserve):
     * epilogue 1 applied to the sum over the group of every rank's y -- a
     * row-parallel projection fused with its all-reduce.  Each rank pushes its
     * rows into every rank's exchange buffer (NVLink stores), counts them on
     * per-row-unit flags, waits (bounded) for all ranks' pushes of the rows it
     * finalises and sums them in rank order, so every rank holds the same h.
     * Consecutive fused calls must alternate exchange_region 0 and 1. */
    int32_t exchange_region;
} affon_b200_qmv_fusion;

int affon_b200_qmv_fused(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                         const void *s, const void *b, void *y, const affon_b200_qmv_fusion *fusion);

/* Residual add and RMSNorm for the tensor-parallel decoder, after the
 * all-reduce of a row-parallel projection: h[m] += add[m] (f32; add may be
 * NULL), then dst[m] = bf16(h[m] * rsqrt(mean(h[m]^2) + eps) * gamma) in the
 * qmv's column order for `bits`.  rows <= 32, cols <= 8192, deterministic. */
int affon_b200_resid_norm(affon_b200_ctx *ctx, float *h, int64_t ld_h, const float *add, int64_t ld_add,
                          const void *gamma, float eps, int rows, int cols, int bits, void *dst, int64_t ld_dst);

/* Grouped-query decode attention over a [batch][kv_heads][capacity][128] bf16
 * KV cache: RoPE (rotate-half pairs, tables [capacity][64]) on the queries
 * and the new key, the new key/value written at *pos, softmax over positions
 * 0..*pos, output [batch][q_heads*128] bf16.  q/k/v are columns q_offset,
 * k_offset, v_offset of the bf16 rows of qkv.  A *pos outside [0, capacity)
 * writes nothing and makes the next affon_b200_ctx_synchronize return
 * AFFON_B200_INVALID_ARG. */
typedef struct affon_b200_attn_desc {
    uint32_t struct_size;
    int32_t batch, q_heads, kv_heads, head_dim, capacity;
    float scale;
    int32_t q_offset, k_offset, v_offset;
    int32_t out_pair_order; /* write the output in 4-bit qmv pair order */
    int64_t ld_qkv, ld_out;
} affon_b200_attn_desc;

int affon_b200_decode_attention(affon_b200_ctx *ctx, const affon_b200_attn_desc *desc, const void *qkv,
                                void *k_cache, void *v_cache, const float *rope_cos, const float *rope_sin,
                                const int *pos, void *out);

/* h[b][:] = f32(table[tokens[b]][:]) with ss_out[dim/16][32] partial sums of
 * squares for the first norm; also zeroes amax[0..batch).  batch <= 32.  A
 * token outside [0, vocab) reads row 0 and makes the next
 * affon_b200_ctx_synchronize return AFFON_B200_INVALID_ARG.  When gamma is
 * given, also x[b][c(k)] = bf16(h[b][k] * gamma[k]) (the first projection's
 * row-scale-mode activations; c in the 4-bit pair order when pair_order). */
int affon_b200_embed(affon_b200_ctx *ctx, const void *table, int64_t ld_table, int64_t vocab, const int *tokens,
                     int batch, int dim, float *h, float *ss_out, unsigned long long *amax, const void *gamma,
                     void *x, int64_t ld_x, int pair_order);

/* tokens[b] = argmax index held in amax[b]; history[*step % history_rows][b]
 * = tokens[b] (history may be NULL; it keeps the last history_rows steps);
 * then *pos += 1 and *step += 1. */
int affon_b200_argmax_finalize(affon_b200_ctx *ctx, const unsigned long long *amax, int batch, int *tokens,
                               int *history, int history_rows, int *pos, int *step);

/* ---------------------------------------------------------------------------
 * Tensor parallelism (whole-model decode sharded over the GPUs of one node,
 * one process per GPU).  No counterpart in the reference, which has no
 * multi-device contract (docs/core/backend-support.md:82); the sharding is
 * column-parallel QKV / gate-up / LM head and row-parallel O / down with a
 * sum all-reduce after each row-parallel projection.  The group is an NCCL
 * communicator attached to a context, created non-blocking: initialisation,
 * every collective's enqueue, affon_b200_tp_synchronize and teardown are
 * polled against a host deadline and abort the group (AFFON_B200_TIMEOUT)
 * instead of hanging on a peer that died or never joined.  Collectives run on
 * the context's stream and can be captured in CUDA graphs. */

#define AFFON_B200_TP_ID_BYTES 144

typedef enum affon_b200_reduce_op {
    AFFON_B200_REDUCE_SUM = 0,
    AFFON_B200_REDUCE_MAX = 1
} affon_b200_reduce_op;

/* A sealed group id (magic, NCCL unique id, checksum) for rank 0 to share
 * with the other ranks out of band (AFFON_B200_TP_ID_BYTES bytes). */
int affon_b200_tp_unique_id(void *id_out);
/* AFFON_B200_OK if `id` is an intact sealed id, else AFFON_B200_INVALID_ARG. */
int affon_b200_tp_id_check(const void *id);
/* Join the group as `rank` of `world` on the context's device; every rank
 * calls it with the same id.  Waits at most timeout_s for all ranks. */
int affon_b200_tp_init(affon_b200_ctx *ctx, int rank, int world, const void *id, double timeout_s);
int affon_b200_tp_rank(const affon_b200_ctx *ctx);   /* -1 without a group */
int affon_b200_tp_world(const affon_b200_ctx *ctx);  /* 0 without a group */
/* Exchange buffers for the fused row-parallel qmv (epilogue 4): two regions
 * of [world][max_rows][max_cols] f32 per rank, mapped by every rank through
 * CUDA IPC (handles gathered over the group).  Collective: every rank calls
 * it with the same sizes. */
int affon_b200_tp_exchange_reserve(affon_b200_ctx *ctx, int max_rows, int64_t max_cols);
/* In-place all-reduce of `count` elements on the context's stream: f32 or
 * bf16 sum, or u64 max. */
int affon_b200_tp_allreduce(affon_b200_ctx *ctx, void *buf, size_t count, int dtype, int op);
int affon_b200_tp_allreduce_bf16(affon_b200_ctx *ctx, void *buf, size_t count);
/* Wait (at most timeout_s; <= 0: the group's) for the context's stream, then
 * report device-side failures like affon_b200_ctx_synchronize. */
int affon_b200_tp_synchronize(affon_b200_ctx *ctx, double timeout_s);
/* Abort the group: peers' pending and future collectives fail. */
int affon_b200_tp_abort(affon_b200_ctx *ctx);
/* Leave the group (bounded finalize, then destroy; abort on timeout). */
int affon_b200_tp_destroy(affon_b200_ctx *ctx);

/* Number of kernel launches this library issued in this process (all
 * contexts); lets callers and benchmarks count native launches. */
uint64_t affon_b200_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* AFFON_B200_H */
