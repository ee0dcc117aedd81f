// Internal launch interfaces shared by the C-ABI layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace afb {

// A resolved operand: device base already offset by the view's byte offset.
struct View {
    const void *ptr;
    int64_t row_stride;
    int64_t col_stride;
};

struct QmmArgs {
    View x, w, s, b;
    void *y;
    int64_t ldy;
    int64_t M, N, K, group;
    int bits;
    int x_bf16, p_bf16, y_bf16;
};

// Generic strided kernel: any bits / group / dtype / view; one thread per
// output element, same operation order as the CPU oracle.
cudaError_t launch_qmm_generic(const QmmArgs &a, cudaStream_t stream);

// Decode qmv for M <= 32, bits in {4, 8}, group 64, bf16 x/s/b, dense rows.
struct QmvPlan {
    int splits;      // K splits (>= 1; 0 = not plannable): x slices that fit shared memory
    int ks;          // K per split
    int grid_n;      // persistent CTAs
    int stages;      // shared-memory ring depth
    int max_slots;   // partial-sum slots per block in the workspace
    int smem_bytes;
    int variant;     // kernel instantiation (activation fragments, tiles per warp, consumer warps)
    int rows;        // weight rows per block
};

// Context workspace layout: [0, 256) device status words (a bounded wait that
// gives up writes there); [kCounterOffset, kPartialOffset) split-K arrival
// counters (first half) and completion counters (second half), zero between
// launches; [kPartialOffset, ...) f32 partial sums.
constexpr size_t kCounterOffset = 256;
// Most activation rows the decode qmv takes in one pass, and the row width of
// the per-16-column sums of squares ([cols/16][kSsWidth] f32) that the
// residual epilogue writes and the RMSNorm prologue reads.
constexpr int kMaxQmvRows = 32;
constexpr int kSsWidth = 32;
// Tensor-parallel exchange: ranks at most, and arrival flags per region.
constexpr int kTpMaxWorld = 8;
constexpr int kTpMaxUnits = 65536;
constexpr int64_t kMaxTiles = 262144;
constexpr size_t kPartialOffset = kCounterOffset + size_t(kMaxTiles) * 4;
// Optional fusions of the decode qmv (decoder use).  Activations: natural
// bf16 x (x_mode 0; 4-bit codes then convert it into the workspace tail) or
// x already in the kernel's column order (x_mode 1, written by
// launch_qmv_prep or by a fused producer).  Epilogues: store y; add into h
// and write per-16-row-tile sums of squares of the new h; silu(gate) * up
// into `act` for weights whose 16-row tiles hold 8 gate rows then the
// matching 8 up rows (optionally in the 4-bit pair order); per-row argmax
// packed as (order-preserving key << 32 | ~n) with atomicMax (lowest index
// wins ties).
// EPI_RESID_AR: EPI_RESID of the sum over the tensor-parallel group of
// every rank's output (a row-parallel projection): the rows are pushed to
// every rank's exchange buffer, and each rank sums the pushes in rank order.
enum QmvEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_SILU_MUL = 2, EPI_ARGMAX = 3, EPI_RESID_AR = 4 };
struct QmvFusion {
    int x_mode = 0;                 // 0: natural bf16 x; 1: x already in the kernel's order
    int epi = EPI_STORE;
    float *h_out = nullptr;         // EPI_RESID: [M][ld_h_out] f32, updated in place
    int64_t ld_h_out = 0;
    float *ss_out = nullptr;        // EPI_RESID: [N/16][16] f32
    uint16_t *act = nullptr;        // EPI_SILU_MUL: [M][ld_act] bf16, N/2 columns
    int64_t ld_act = 0;
    int act_pair_order = 0;         // EPI_SILU_MUL: write act in the 4-bit pair order
    unsigned long long *amax = nullptr;  // EPI_ARGMAX: [M]
    int64_t index_offset = 0;       // EPI_ARGMAX: added to the row index (a vocabulary shard's first row)
    // Row-scale mode: x is bf16(h * gamma) (not normalised); every output of
    // activation row m is multiplied by rsqrt(sum_k h[m][k]^2 / K + eps),
    // with the sums of squares taken from row_ss ([ss_tiles][kSsWidth]).
    const float *row_ss = nullptr;
    int ss_tiles = 0;
    float eps = 0.0f;
    // EPI_RESID: also write next_x[m][col(n)] = bf16(h_new[m][n] * next_gamma[n])
    // (the next projection's row-scale-mode activations; col in pair order
    // when next_pair_order).
    const uint16_t *next_gamma = nullptr;
    uint16_t *next_x = nullptr;
    int64_t ld_next_x = 0;
    int next_pair_order = 0;
    // EPI_RESID_AR: every rank's receive area ([world][M][N] f32) and arrival
    // flags of this call's exchange region.
    int tp_world = 1, tp_rank = 0;
    float *tp_recv[kTpMaxWorld] = {};
    unsigned *tp_flags_peer[kTpMaxWorld] = {};
    unsigned *tp_flags_local = nullptr;
};
bool qmv_supported(const QmmArgs &a, const char **why);
// allow_ws = false keeps to the stream-K kernel (the tensor-parallel fused
// exchange, whose multi-GPU runs cover that kernel).
QmvPlan qmv_plan(const QmmArgs &a, int num_sms, size_t workspace_bytes, bool allow_ws = true);
size_t qmv_workspace_bytes(const QmmArgs &a, const QmvPlan &p);
// Bytes at the end of the qmv workspace that hold pair-ordered x (4-bit, x_mode 0).
size_t qmv_prep_bytes(const QmmArgs &a);
// Activations into the qmv's order (4-bit: pair order [x0 x4 x1 x5 x2 x6 x3 x7]
// within every 8 columns; 8-bit: natural), bf16 [M][ld_dst].  mode 0: src is
// bf16 [M][ld_src]; mode 1: src is the f32 residual stream h, normalised with
// the per-16-column partial sums of squares ss ([ss_tiles][16]) and gamma.
cudaError_t launch_qmv_prep(const void *src, int64_t ld_src, int mode, const float *ss, int ss_tiles,
                            const uint16_t *gamma, float eps, int M, int K, int bits, uint16_t *dst, int64_t ld_dst,
                            cudaStream_t stream, bool pdl = false);
// pdl: launch with programmatic dependent launch (the kernel prefetches its
// weights before waiting for the preceding kernel in the stream).
cudaError_t launch_qmv(const QmmArgs &a, const QmvPlan &p, void *workspace, cudaStream_t stream,
                       const QmvFusion *fusion = nullptr, bool pdl = false);
// h[m] += add[m] (add may be null), then dst[m] = bf16(rmsnorm(h[m]) * gamma)
// in the qmv's column order for `bits`; one CTA per row, K <= 8192.
cudaError_t launch_resid_norm(float *h, int64_t ld_h, const float *add, int64_t ld_add, const uint16_t *gamma,
                              float eps, int M, int K, int bits, uint16_t *dst, int64_t ld_dst, cudaStream_t stream,
                              bool pdl);
// Test hook of the split-K combine: its wait limit (0 = the default) and
// arrivals it waits for beyond the real contributors (0 in normal use; 1
// makes every shared block's wait run out).  Process-wide.
void qmv_set_combine_wait(uint64_t limit_ns, unsigned extra_arrivals);

// Decoder kernels around the quantized linears (decode.cu).
struct DecodeAttnArgs {
    const void *qkv;
    int64_t ld_qkv;
    int q_off, k_off, v_off;
    void *k_cache, *v_cache;        // [batch][kv_heads][capacity][head_dim] bf16
    const float *rope_cos, *rope_sin;  // [capacity][head_dim/2]
    const int *pos;                 // device scalar: position of the new token
    void *out;                      // [batch][q_heads*head_dim] bf16
    int64_t ld_out;
    int batch, q_heads, kv_heads, head_dim, capacity;
    float scale;
    int out_pair_order;             // write out in the 4-bit qmv pair order
};
// Context splits per (batch row, KV head) and the workspace the attention's
// split records need (f32, after kPartialOffset).
int attention_splits(int batch, int kv_heads, int capacity, int num_sms);
size_t attention_workspace_bytes(int batch, int kv_heads, int q_heads, int capacity, int num_sms);
cudaError_t launch_decode_attention(const DecodeAttnArgs &a, void *workspace, int num_sms, cudaStream_t stream,
                                    bool pdl);
cudaError_t launch_embed(const void *table, int64_t ld_table, int64_t vocab, const int *tokens, int B, int D,
                         float *h, float *ss_out, unsigned long long *amax, const uint16_t *gamma, uint16_t *x,
                         int64_t ld_x, int pair_order, void *workspace, cudaStream_t stream, bool pdl);
cudaError_t launch_finalize(const unsigned long long *amax, int B, int *tokens, int *history, int history_rows,
                            int *pos, int *step, cudaStream_t stream, bool pdl);

// Prefill qmm on tcgen05 tensor cores (M >= 64), bf16 x/s/b, 4/8-bit, group 64.
bool qmm_tc_supported(const QmmArgs &a, const char **why);
cudaError_t launch_qmm_tc(const QmmArgs &a, void *workspace, cudaStream_t stream);

// Prefill qmm with reassociated numerics on tcgen05 tensor cores (M >= 64,
// bf16 x/s/b, 4/8-bit, group 64): exact codes, per-group f32 scales, the bias
// term as a tensor-core product with exact bf16 pieces of the group sums.
// Needs at least qmm_exact_min_workspace(a) bytes of workspace; larger M is
// processed in row slices that fit.
bool qmm_exact_supported(const QmmArgs &a, const char **why);
size_t qmm_exact_min_workspace(const QmmArgs &a);
cudaError_t launch_qmm_exact(const QmmArgs &a, void *workspace, size_t workspace_bytes, cudaStream_t stream);
void qmm_exact_set_slice_cap(int64_t rows);  // test hook: most rows per pass (0 = workspace bound)

void count_launch(uint64_t n = 1);

}  // namespace afb

struct affon_b200_qmm_desc;

namespace afb {
struct TpState;
}

// A context: one device, one stream, a workspace, and (after
// affon_b200_tp_init) its place in a tensor-parallel group.
struct affon_b200_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    bool overlap = false;  // programmatic dependent launch for the decode kernels
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
    // Staging buffers of the host-buffer entry points (grown on demand).
    void *stage[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    size_t stage_bytes[5] = {0, 0, 0, 0, 0};
    afb::TpState *tp = nullptr;
};

namespace afb {
// Tears down the context's tensor-parallel state (tp.cu).
void tp_release(affon_b200_ctx *ctx);
// Fill f's exchange fields for a row-parallel qmv of `rows` x `cols` outputs
// with `units` row units, using exchange region `region` (0 or 1).
bool tp_bind_exchange(affon_b200_ctx *ctx, int region, int64_t rows, int64_t cols, int64_t units, QmvFusion *f,
                      const char **why);
// Descriptor validation, argument resolution and the thread-local error
// message of the C ABI (abi.cu), for other entry points of the library.
int validate_qmm_desc(const affon_b200_qmm_desc *d);
QmmArgs qmm_args_from_desc(const affon_b200_qmm_desc *d, const void *x, const void *w, const void *s, const void *b,
                           void *y);
int set_error(int status, const char *msg);
int set_cuda_error(cudaError_t e, const char *what);
void clear_error();

}  // namespace afb
