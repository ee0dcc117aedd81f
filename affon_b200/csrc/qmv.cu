// Decode qmv for sm_100a: y[M,N] = x[M,K] . decode(W)[N,K]^T for M <= 32,
// 4- or 8-bit codes packed little-endian into u32 along K, group 64, bf16
// activations / scales / biases, f32 accumulation (the layout and formula of
// docs/core/quantized-inference.md:45-67).
//
// Streaming.  Persistent CTAs, one per SM.  One producer warp moves each
// block-row x 128-byte stage of the packed weight matrix through a ring of
// shared-memory stages with 2D TMA loads (128-byte swizzle), together with the
// matching boxes of bf16 scales and biases (8 groups wide) and the stage's
// activation columns (16 or 32 rows x 64 columns per group, 128-byte swizzle;
// one 3D box per stage).
// The ring holds ~190 KB per SM in flight without costing registers, and the
// activations need no separate staging pass.  Twelve consumer warps decode the
// packed words in registers and feed tensor cores: for M <= 16 each warp owns
// two 16-row weight tiles (384-row blocks), so each activation fragment feeds
// two tiles; for 16 < M <= 32 one tile (192-row blocks) with four 8-row
// activation fragments.
//
// Overlap with the preceding kernel.  With programmatic dependent launch
// (the context's overlap mode) a CTA may start while the kernel before it in
// the stream is still finishing: the producer fills the first ring stages
// with weights, scales and biases -- which no preceding kernel writes in that
// mode -- and only then waits for the preceding kernel (griddepcontrol.wait)
// before loading activations; every other warp waits before touching any
// global memory.  Each CTA also lets the following kernel launch as soon as it
// starts; the following kernel can then only take SMs this grid leaves idle or
// has finished with, and all CTAs of this grid are already resident.
//
// Why mma.sync tensor cores at M <= 16: at ~6.5 TB/s a 4-bit weight stream
// delivers ~13e12 weights/s; decoding each weight to a float and multiplying
// it on the CUDA cores costs ~3 lane-ops, as much as the 148 SMs can issue.
// The decoded codes go straight from registers into the A fragments of
// m16n8k16 bf16 MMAs (weights as the 16-row A operand, activations as B).
// tcgen05 MMAs do not fit this shape: each instruction occupies the SM's
// tensor core for ~146 cycles whatever its N (16..256), so at N <= 16 the
// 128 x 16 weights per instruction cap a CTA near 7 bytes of codes per cycle.
//
// Exact codes, per-group affine in f32: the MMA multiplies the integer codes
// (4-bit: as 128+q, exact in bf16) by x, giving C_g = sum_{k in g} x*code in
// f32.  The activation sums X_g = sum_{k in g} x[k] are the same for every
// weight row: one "sum" warp per CTA computes them once per stage (MMAs with
// an all-ones A operand) into shared memory.  The affine decode is applied per
// group of 64 outside the tensor core:
//     y += s[n,g] * C_g + (b[n,g] - 128 s[n,g]) * X_g
// with packed f32x2 fused multiply-adds, so the offset terms cancel exactly.
// This is sum_k x*(s*q+b) up to reassociation; weights are never rounded to
// bf16 (quantized-inference.md:119-121).  Numerical class: reassociated.
//
// Activation layout.  For 4-bit codes the kernel reads x in "pair order":
// within every 8 consecutive columns the order is [x0 x4 x1 x5 x2 x6 x3 x7],
// matching the (q_p, q_{p+4}) pairs one logic op extracts from a packed word.
// launch_qmv_prep writes that order from natural bf16 x (and, for the decoder,
// the RMS-normalised residual stream); 8-bit codes use natural order.
//
// Work partition (stream-K).  The work is a flat list of items (384-row
// block, 128-byte K stage).  CTA c takes the items [c*T/C, (c+1)*T/C), so
// every CTA streams the same number of bytes (the grid is the fewest CTAs
// with the makespan of one CTA per SM).  A block that lies inside one CTA is
// stored directly; a block shared by several CTAs is combined through f32
// partials: each contributing CTA writes its slot and counts its arrival on
// the block's counter.  The launch is cooperative (all CTAs resident), so at
// the end every contributor waits (bounded) for the block's count, then sums
// the slots in slot order for its own share of the block's rows and applies
// the epilogue; results do not depend on scheduling.  The last CTA to finish
// a block resets its counters for the next launch.
#include <algorithm>
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace afb {
namespace qmv {

constexpr int GROUP = 64;
constexpr int MAX_STAGES = 8;
constexpr int MAX_WS_STAGES = 20;  // ring depth of the warp-split kernel, at most
constexpr int MAX_XR = 32;             // activation rows staged per group, at most

// Consumer warps (CW), 16-row weight tiles per consumer warp (NT) and 8-row
// activation fragments (MT) of one instantiation; a block is the CTA-wide
// row tile (CW * NT * 16 rows), loaded as NT TMA boxes of CW * 16 rows.
// The register file of each of the SM's four sub-partitions (16K registers)
// holds a quarter of the CTA's warps, rounded up: 14 warps (12 consumers)
// allow 128 registers per thread, 12 warps (10 consumers) 168, which the
// M > 8 variants need to keep their accumulators out of local memory.
template <int BITS, int MT, int NT, int CW>
struct Shape {
    static constexpr int THREADS = 32 * (CW + 2);     // consumers, producer, sum warp
    static constexpr int ROWS = 16 * NT * CW;         // weight rows per block
    static constexpr int BOX_ROWS = 16 * CW;          // TMA box height for weights, scales and biases
    static constexpr int XR = MT == 4 ? 32 : 16;      // activation rows per staged box
    static constexpr int X_BOX = XR * 128;            // one group of activation columns: XR rows x 64 bf16
    static constexpr int GPS = BITS == 4 ? 4 : 2;     // groups per stage (128 packed bytes per row)
    static constexpr int KPS = GPS * GROUP;           // K per stage
    static constexpr int W = ROWS * 128;              // packed bytes per stage
    static constexpr int SB = (ROWS * 16 + 511) / 512 * 512;  // one 8-group box of scales (or biases), padded
    static constexpr int X = GPS * X_BOX;
    static constexpr int BYTES = W + 2 * SB + X;      // swizzled regions (W, X) stay 1024-byte aligned
    static constexpr int TX_BYTES = W + 2 * ROWS * 16 + X;  // bytes the stage's TMA loads deliver (no padding)
    static_assert(W % 1024 == 0 && (2 * SB) % 1024 == 0 && X % 1024 == 0 && BOX_ROWS <= 256, "stage layout");
};

// Instantiations (variant: MT, NT, CW -> block rows): M <= 8: 0 = (1, 2, 12)
// -> 384, 1 = (1, 1, 12) -> 192; M <= 16: 2 = (2, 2, 10) -> 320, 3 = (2, 1, 10)
// -> 160, 5 = (2, 1, 13) -> 208 (whole-K blocks, one per CTA); M <= 32: 4 =
// (4, 1, 10) -> 160.  The planner picks, per shape, the variant with the
// smallest estimated makespan.  Variants 6, 7, 8: the warp-split whole-K
// kernel (qmv_ws_kernel) with T = 1, 2, 3 tiles -> 16, 32, 48 rows, M <= 16.
constexpr int kVariantRows[9] = {384, 192, 320, 160, 160, 208, 16, 32, 48};
constexpr int kVariantNT[9] = {2, 1, 2, 1, 1, 1, 1, 1, 1};
constexpr int kVariantBoxRows[9] = {192, 192, 160, 160, 160, 208, 16, 32, 48};  // one box per block row tile set
static_assert(Shape<4, 1, 2, 12>::BOX_ROWS == kVariantBoxRows[0] && Shape<4, 1, 1, 12>::BOX_ROWS == kVariantBoxRows[1] &&
                  Shape<4, 2, 2, 10>::BOX_ROWS == kVariantBoxRows[2] && Shape<4, 2, 1, 10>::BOX_ROWS == kVariantBoxRows[3] &&
                  Shape<4, 4, 1, 10>::BOX_ROWS == kVariantBoxRows[4] && Shape<4, 2, 1, 13>::BOX_ROWS == kVariantBoxRows[5],
              "tensor-map boxes match the kernels' boxes");

struct Params {
    void *y;
    int64_t ldy;
    float *partial;
    unsigned *counters;
    unsigned *status;
    int M, N, K;
    int nblocks, spb;     // blocks along N and stages per block
    int64_t items;        // nblocks * spb
    int stages;           // ring depth
    int max_slots;        // partial slots per block
    int y_bf16;
    uint64_t arrival_wait_ns;  // limit of the combine's wait for the other contributors
    unsigned extra_arrivals;   // test hook: contributors the combine waits for beyond the real ones (0)
    QmvFusion f;
};

// Codes p and p+4 of a 4-bit word as the exact bf16 pair (128+q_p, 128+q_{p+4}):
// one shift and one logic op.
__device__ __forceinline__ uint32_t dec4(uint32_t w, int p) {
    return lop3_and_or(p ? (w >> (4 * p)) : w, 0x000F000Fu, 0x43004300u);
}
// Bytes i and i+1 of an 8-bit word as an exact bf16 pair (via 2^23 + q in f32).
__device__ __forceinline__ uint32_t dec8(uint32_t w, int i) {
    float f0 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i)) - 8388608.0f;
    float f1 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i + 1)) - 8388608.0f;
    return pack_bf16x2(f0, f1);
}

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
// d = a * b + c on packed f32 pairs (one instruction, sm_100a).
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ void store_out(const Params &p, int m, int64_t n, float v) {
    if (p.y_bf16)
        static_cast<uint16_t *>(p.y)[m * p.ldy + n] = f32_to_bf16_bits(v);
    else
        static_cast<float *>(p.y)[m * p.ldy + n] = v;
}

// Owner CTA of flat item i when CTA c holds [floor(c*T/C), floor((c+1)*T/C)).
__device__ __forceinline__ int owner_of(int64_t i, int64_t T, int C) {
    return static_cast<int>(((i + 1) * C - 1) / T);
}

__device__ __forceinline__ uint32_t f32_order_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Pair-order slot of column e (0..7) within its 8 columns: 0 4 1 5 2 6 3 7.
__device__ __forceinline__ int pair_slot(int e) { return (e < 4) ? 2 * e : 2 * (e - 4) + 1; }

// Apply the epilogue to the row pair (n_lo, n_lo + 8) of activation row m.
// Returns the contribution of this pair to the per-tile reductions:
// EPI_RESID: sum of squares of the updated residual entries; EPI_ARGMAX: the
// packed best (key << 32 | ~n) of the pair.  Rows at or beyond N are skipped.
// Residual update of one element: h += v, the next projection's
// activation bf16(h * gamma_next) at its column-order position when asked,
// and the square for the sums of squares.
// h_pre / g_pre: h[m][n] and next_gamma[n] already loaded by the caller
// (their loads issued together with the caller's other loads).
__device__ __forceinline__ float resid_update(const Params &p, int m, int64_t n, float v, float &ssq,
                                              const float *h_pre = nullptr, const float *g_pre = nullptr) {
    float *h = p.f.h_out + m * p.f.ld_h_out;
    const float hv = (h_pre ? *h_pre : h[n]) + v;
    h[n] = hv;
    if (p.f.next_x) {
        const int e = static_cast<int>(n & 7);
        const int64_t col = p.f.next_pair_order ? (n & ~int64_t(7)) + pair_slot(e) : n;
        const float gm = g_pre ? *g_pre : bf16_bits_to_f32(p.f.next_gamma[n]);
        p.f.next_x[m * p.f.ld_next_x + col] = f32_to_bf16_bits(hv * gm);
    }
    ssq = fmaf(hv, hv, ssq);
    return hv;
}

// EPI_RESID_AR: this rank's value of output (m, n) into every rank's receive
// area, at this rank's slot (plain stores; the peers' areas are NVLink
// mappings).
__device__ __forceinline__ void ar_push(const Params &p, int m, int64_t n, float v) {
    const int64_t off = (static_cast<int64_t>(p.f.tp_rank) * p.M + m) * p.N + n;
#pragma unroll
    for (int r = 0; r < kTpMaxWorld; ++r)
        if (r < p.f.tp_world) p.f.tp_recv[r][off] = v;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *a) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}

// EPI_RESID_AR: after the consumer warps pushed the rows of one unit (a
// whole block, or this CTA's share of a shared block), count the unit's
// arrival on every rank: the CTA barrier orders every thread's pushes before
// thread 0's system-scope fence (cumulative), which orders them before its
// increments of the peers' flags.  Called by all consumer threads.
template <int CW>
__device__ __forceinline__ void ar_signal(const Params &p, int unit, int tid) {
    named_bar_sync(1, CW * 32);
    if (tid == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int r = 0; r < p.f.tp_world; ++r)
            asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(p.f.tp_flags_peer[r] + unit) : "memory");
    }
}

// pre (EPI_RESID): h[m][n_lo], h[m][n_hi], next_gamma[n_lo], next_gamma[n_hi]
// already loaded by the caller.
__device__ __forceinline__ unsigned long long epilogue_pair(const Params &p, int m, int64_t n_lo, float v_lo,
                                                            float v_hi, float &ssq, const float *rs,
                                                            const float *pre = nullptr) {
    const int64_t n_hi = n_lo + 8;
    const bool ok_lo = n_lo < p.N, ok_hi = n_hi < p.N;
    unsigned long long best = 0ull;
    if (rs) {  // RMSNorm scale of the (unnormalised) activation row
        v_lo *= rs[m];
        v_hi *= rs[m];
    }
    switch (p.f.epi) {
    case EPI_RESID: {
        const bool g = pre && p.f.next_x;
        if (ok_lo) resid_update(p, m, n_lo, v_lo, ssq, pre ? &pre[0] : nullptr, g ? &pre[2] : nullptr);
        if (ok_hi) resid_update(p, m, n_hi, v_hi, ssq, pre ? &pre[1] : nullptr, g ? &pre[3] : nullptr);
        break;
    }
    case EPI_RESID_AR:
        if (ok_lo) ar_push(p, m, n_lo, v_lo);
        if (ok_hi) ar_push(p, m, n_hi, v_hi);
        break;
    case EPI_SILU_MUL:
        if (ok_hi) {  // tile rows 0-7 are gate rows, 8-15 the matching up rows
            // act column j = 8*(n/16) + n%8, at its pair-order slot when the
            // consumer is a 4-bit qmv
            const int e = static_cast<int>(n_lo & 7);
            const int64_t j = (n_lo >> 4) * 8 + (p.f.act_pair_order ? pair_slot(e) : e);
            const float gate = v_lo;
            const float silu = gate / (1.0f + __expf(-gate));
            p.f.act[m * p.f.ld_act + j] = f32_to_bf16_bits(silu * v_hi);
        }
        break;
    case EPI_ARGMAX: {
        const int64_t off = p.f.index_offset;
        if (ok_lo)
            best = (static_cast<unsigned long long>(f32_order_key(v_lo)) << 32) | (0xFFFFFFFFu - uint32_t(n_lo + off));
        if (ok_hi) {
            const unsigned long long c =
                (static_cast<unsigned long long>(f32_order_key(v_hi)) << 32) | (0xFFFFFFFFu - uint32_t(n_hi + off));
            best = c > best ? c : best;
        }
        break;
    }
    default:
        if (ok_lo) store_out(p, m, n_lo, v_lo);
        if (ok_hi) store_out(p, m, n_hi, v_hi);
    }
    return best;
}

// Reduce a per-pair value over the 8 lanes that share t (lanes t, t+4, ...)
// and publish it once per (tile, m): sums of squares go to ss_out[tile][m],
// argmax candidates to amax[m].
__device__ __forceinline__ void publish_tile(const Params &p, int64_t tile, int m, bool lead, float ssq,
                                             unsigned long long best) {
    if (p.f.epi == EPI_RESID) {
        ssq += __shfl_xor_sync(0xffffffffu, ssq, 4);
        ssq += __shfl_xor_sync(0xffffffffu, ssq, 8);
        ssq += __shfl_xor_sync(0xffffffffu, ssq, 16);
        if (lead && m < p.M) p.f.ss_out[tile * kSsWidth + m] = ssq;
    } else if (p.f.epi == EPI_ARGMAX) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lead && m < p.M && best) atomicMax(&p.f.amax[m], best);
    }
}

// Final values of one thread for one 16-row tile: rows n0+g and n0+g+8,
// activation rows 2t, 2t+1 (+8 for the second MMA column tile).  Called by
// all 32 lanes of the warp.
// Residual-epilogue operands of one thread for one 16-row tile (finish_tile's
// layout): pre[mt][h] = {h[m][n], h[m][n+8], gamma[n], gamma[n+8]} for
// activation row m = 2t + 8mt + h and weight rows n = n0 + g, n0 + g + 8.
template <int MT>
__device__ __forceinline__ void load_resid_operands(const Params &p, int64_t n0, int g, int t, float (&pre)[MT][2][4]) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = 2 * t + 8 * mt + h;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int64_t n = n0 + g + 8 * e;
                const bool ok = m < p.M && n < p.N;
                pre[mt][h][e] = ok ? p.f.h_out[m * p.f.ld_h_out + n] : 0.0f;
                pre[mt][h][2 + e] = ok && p.f.next_x ? bf16_bits_to_f32(p.f.next_gamma[n]) : 0.0f;
            }
        }
}

template <int MT>
__device__ __forceinline__ void finish_tile(const Params &p, const float (&v)[MT][4], int64_t n0, int g, int t,
                                            const float *rs, const float (*pre_in)[2][4] = nullptr) {
    // The residual epilogue reads h and the next norm's weights: issue all of
    // this thread's loads before its first store (one round trip, not one per
    // element), unless the caller fetched them earlier (pre_in).
    float pre[MT][2][4];
    const bool resid = p.f.epi == EPI_RESID;
    if (resid && pre_in) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 4; ++e) pre[mt][h][e] = pre_in[mt][h][e];
    } else if (resid) {
        load_resid_operands<MT>(p, n0, g, t, pre);
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = 2 * t + 8 * mt + h;
            float ssq = 0.0f;
            unsigned long long best = 0ull;
            if (m < p.M) best = epilogue_pair(p, m, n0 + g, v[mt][h], v[mt][2 + h], ssq, rs, resid ? pre[mt][h] : nullptr);
            publish_tile(p, n0 >> 4, m, g == 0, ssq, best);
        }
}

// Final value v of weight row n for activation row m, one thread per row,
// 32 consecutive rows per warp (a 16-row tile is one half warp; rows n and
// n+8 sit in lanes l and l+8).  Called by all 32 lanes with the same m.
// Residual update of rows n (one per lane, 32 consecutive rows per warp,
// the same m) with the per-16-row sums of squares.  Called by all 32 lanes.
__device__ __forceinline__ void resid_row(const Params &p, int m, int64_t n, float v, int lane, bool ok,
                                          const float *h_pre = nullptr, const float *g_pre = nullptr) {
    float ssq = 0.0f;
    if (ok) resid_update(p, m, n, v, ssq, h_pre, g_pre);
    ssq += __shfl_xor_sync(0xffffffffu, ssq, 1);
    ssq += __shfl_xor_sync(0xffffffffu, ssq, 2);
    ssq += __shfl_xor_sync(0xffffffffu, ssq, 4);
    ssq += __shfl_xor_sync(0xffffffffu, ssq, 8);
    if (ok && (lane & 15) == 0) p.f.ss_out[(n >> 4) * kSsWidth + m] = ssq;
}

__device__ __forceinline__ void finish_row(const Params &p, int m, int64_t n, float v, int lane, bool active,
                                           const float *rs, const float *h_pre = nullptr,
                                           const float *g_pre = nullptr) {
    const bool ok = active && n < p.N;
    if (rs) v *= rs[m];
    switch (p.f.epi) {
    case EPI_RESID:
        resid_row(p, m, n, v, lane, ok, h_pre, g_pre);
        break;
    case EPI_RESID_AR:
        if (ok) ar_push(p, m, n, v);
        break;
    case EPI_SILU_MUL: {
        const float up = __shfl_down_sync(0xffffffffu, v, 8);
        if (active && (lane & 8) == 0 && n + 8 < p.N) {
            const int e = static_cast<int>(n & 7);
            const float silu = v / (1.0f + __expf(-v));
            p.f.act[m * p.f.ld_act + (n >> 4) * 8 + (p.f.act_pair_order ? pair_slot(e) : e)] =
                f32_to_bf16_bits(silu * up);
        }
        break;
    }
    case EPI_ARGMAX: {
        unsigned long long best =
            ok ? (static_cast<unsigned long long>(f32_order_key(v)) << 32) | (0xFFFFFFFFu - uint32_t(n + p.f.index_offset))
               : 0ull;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0 && best) atomicMax(&p.f.amax[m], best);
        break;
    }
    default:
        if (ok) store_out(p, m, n, v);
    }
}

// Contributors of block blk: CTAs first..first+total-1 (stream-K ranges).
__device__ __forceinline__ void block_contributors(const Params &p, int blk, int &first, int &total) {
    const int64_t b0 = static_cast<int64_t>(blk) * p.spb;
    first = owner_of(b0, p.items, gridDim.x);
    total = owner_of(b0 + p.spb - 1, p.items, gridDim.x) - first + 1;
}

// End of one block segment of this CTA, called by all consumer warps
// together.  A block inside one CTA is finished here.  Otherwise the CTA
// writes its f32 partial slot and announces it on the block's arrival
// counter; the sums are formed in combine_blocks once every contributor has
// written its slot.
template <int MT, int NT, int CW>
__device__ __forceinline__ void segment_epilogue(const Params &p, const float (&acc)[NT][MT][4], int blk, int warp,
                                                 int g, int t, int tid, const float *rs, uint64_t *rsbar,
                                                 volatile int *abort) {
    constexpr int CT = CW * 32;  // consumer threads
    constexpr int ROWS = 16 * NT * CW;
    int first, total;
    block_contributors(p, blk, first, total);
    const int64_t nb0 = static_cast<int64_t>(blk) * ROWS;
    if (total == 1) {
        if (rs) mbar_wait(rsbar, 0, abort, p.status);  // the row scales are out
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) finish_tile<MT>(p, acc[nt], nb0 + (warp * NT + nt) * 16, g, t, rs);
        if (p.f.epi == EPI_RESID_AR) ar_signal<CW>(p, blk * p.max_slots, tid);
        return;
    }
    const int slot = static_cast<int>(blockIdx.x) - first;
    // partial[((blk * max_slots + slot) * M + m) * ROWS + row]
    float *base = p.partial + static_cast<int64_t>(blk) * p.max_slots * p.M * ROWS;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = 2 * t + 8 * mt + (i & 1);
                const int r = (warp * NT + nt) * 16 + g + 8 * (i >> 1);
                if (m < p.M) base[(static_cast<int64_t>(slot) * p.M + m) * ROWS + r] = acc[nt][mt][i];
            }
    // Release: every thread orders its partial stores at gpu scope, the
    // consumer warps meet, and one thread counts the CTA's arrival.
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    named_bar_sync(1, CT);
    if (tid == 0) atomicAdd(&p.counters[blk], 1u);
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *a) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}

// One block this CTA shares with other contributors: its slot and this
// CTA's share of the block's 16-row tiles.
struct SharedBlock {
    int blk, slot, total, row0, nrows, units;
};

template <int ROWS>
__device__ __forceinline__ SharedBlock shared_block(const Params &p, int blk) {
    constexpr int TILES = ROWS / 16;
    SharedBlock b;
    int first;
    block_contributors(p, blk, first, b.total);
    b.blk = blk;
    b.slot = static_cast<int>(blockIdx.x) - first;
    const int t0 = b.slot * TILES / b.total, t1 = (b.slot + 1) * TILES / b.total;
    b.row0 = t0 * 16;
    b.nrows = (t1 - t0) * 16;
    b.units = ((b.nrows + 31) / 32) * p.M;
    return b;
}

// Second phase (every CTA of the grid is resident).  Only the first and the
// last block of a CTA's range can be shared with other CTAs (every block in
// between lies inside the range).  For those, wait until all contributors
// have published their slots, then sum the slots in slot order for this
// CTA's share of each block's 16-row tiles and apply the epilogue -- both
// blocks in one pass, so their slot loads travel together.  The CTA finishing
// a block last resets its counters for the next launch.  The waits are
// bounded; on timeout the status word says TIMEOUT and the CTA goes on (its
// results are then garbage, and the counters are still reset).
template <int ROWS, int CW>
__device__ void combine_blocks(const Params &p, int64_t lo, int64_t hi, int warp, int lane, int tid,
                               volatile int *abort, const float *rs, uint64_t *rsbar) {
    // Units per batch: three where the 168-register variants have room, two in
    // the 128-register ones; slots per unit loaded together: MAXS.
    constexpr int CT = CW * 32, UB = CW == 10 ? 3 : 2, MAXS = 16;
    if (hi <= lo) return;
    unsigned *done = p.counters + kMaxTiles / 2;
    const int b_first = static_cast<int>(lo / p.spb), b_last = static_cast<int>((hi - 1) / p.spb);
    SharedBlock A = shared_block<ROWS>(p, b_first), B = shared_block<ROWS>(p, b_last);
    const bool hasA = A.total > 1, hasB = b_last != b_first && B.total > 1;
    if (!hasA && !hasB) return;
    if (!hasA) {  // B alone: keep it in the first place
        A = B;
    }
    const bool two = hasA && hasB;
    if (!two) B.units = 0;
    if (tid == 0) {
        const uint64_t start = globaltimer();
        for (int k = 0; k < (two ? 2 : 1); ++k) {
            const SharedBlock &sb = k == 0 ? A : B;
            const unsigned want = static_cast<unsigned>(sb.total) + p.extra_arrivals;
            while (ld_acquire_gpu(&p.counters[sb.blk]) < want) {
                if (*abort || globaltimer() - start > p.arrival_wait_ns) {
                    *abort = 1;
                    atomicExch(p.status, static_cast<unsigned>(DEV_TIMEOUT));
                    break;
                }
                __nanosleep(64);
            }
        }
    }
    named_bar_sync(1, CT);
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (rs) mbar_wait(rsbar, 0, abort, p.status);  // the row scales are out
    const int64_t slot_stride = static_cast<int64_t>(p.M) * ROWS;
    const float *baseA = p.partial + static_cast<int64_t>(A.blk) * p.max_slots * slot_stride;
    const float *baseB = p.partial + static_cast<int64_t>(B.blk) * p.max_slots * slot_stride;
    const int units = A.units + B.units;
    const bool resid = p.f.epi == EPI_RESID, gamma = resid && p.f.next_x != nullptr;
    // Work unit = (block, 32-row chunk, activation row m), one warp each; a
    // warp takes UB units at a time and issues every load of all of them --
    // up to MAXS slots each, and the residual row and next-norm weights the
    // residual epilogue reads -- before summing, so a batch costs about one
    // L2 round trip.
    for (int ub = warp; ub < units; ub += CW * UB) {
        float part[UB][MAXS], hpre[UB], gpre[UB];
#pragma unroll
        for (int u = 0; u < UB; ++u) {
            const int unit = ub + u * CW;
            const bool inB = unit >= A.units;
            const int local = unit < units ? (inB ? unit - A.units : unit) : 0;
            const int chunk = local / p.M, m = local - chunk * p.M;
            const int rr = chunk * 32 + lane;
            const int nrows = inB ? B.nrows : A.nrows, total = inB ? B.total : A.total;
            const int row = (inB ? B.row0 : A.row0) + (rr < nrows ? rr : 0);
            const float *src = (inB ? baseB : baseA) + static_cast<int64_t>(m) * ROWS + row;
#pragma unroll
            for (int k = 0; k < MAXS; ++k) part[u][k] = (k < total && unit < units) ? __ldcg(src + k * slot_stride) : 0.0f;
            const int64_t n = static_cast<int64_t>(inB ? B.blk : A.blk) * ROWS + row;
            const bool ok = resid && unit < units && rr < nrows && n < p.N;
            hpre[u] = ok ? p.f.h_out[m * p.f.ld_h_out + n] : 0.0f;
            gpre[u] = ok && gamma ? bf16_bits_to_f32(p.f.next_gamma[n]) : 0.0f;
        }
        // Slots beyond MAXS (more than MAXS contributors) are added after.
#pragma unroll
        for (int u = 0; u < UB; ++u) {
            const int unit = ub + u * CW;
            if (unit >= units) break;  // warp-uniform
            const bool inB = unit >= A.units;
            const int local = inB ? unit - A.units : unit;
            const int chunk = local / p.M, m = local - chunk * p.M;
            const int rr = chunk * 32 + lane;
            const int nrows = inB ? B.nrows : A.nrows, total = inB ? B.total : A.total;
            const int row0 = inB ? B.row0 : A.row0, blk = inB ? B.blk : A.blk;
            const bool active = rr < nrows;
            const int row = row0 + (active ? rr : 0);
            const float *src = (inB ? baseB : baseA) + static_cast<int64_t>(m) * ROWS + row;
            float v = 0.0f;
#pragma unroll
            for (int k = 0; k < MAXS; ++k)
                if (k < total) v += part[u][k];
            for (int k = MAXS; k < total; ++k) v += __ldcg(src + k * slot_stride);
            finish_row(p, m, static_cast<int64_t>(blk) * ROWS + row0 + rr, v, lane, active, rs, resid ? &hpre[u] : nullptr,
                       gamma ? &gpre[u] : nullptr);
        }
    }
    for (int k = 0; k < (two ? 2 : 1); ++k) {
        const SharedBlock &sb = k == 0 ? A : B;
        if (p.f.epi == EPI_RESID_AR) ar_signal<CW>(p, sb.blk * p.max_slots + sb.slot, tid);
        if (tid == 0 && atomicAdd(&done[sb.blk], 1u) == static_cast<unsigned>(sb.total - 1)) {
            p.counters[sb.blk] = 0u;
            done[sb.blk] = 0u;
        }
    }
}

// EPI_RESID_AR, last phase: wait (bounded) until every rank has pushed the
// rows of every unit this CTA finalised, then sum them in rank order and apply
// the residual update.  Every rank finalises the same units with the same
// plan, so a unit's flag reaches the world size exactly once per launch; the
// waiter resets it (no rank touches it again in this launch).
template <int ROWS, int CW>
__device__ void ar_finish(const Params &p, int64_t lo, int64_t hi, int warp, int lane, int tid, volatile int *abort) {
    constexpr int CT = CW * 32, TILES = ROWS / 16;
    if (hi <= lo) return;
    const int b_first = static_cast<int>(lo / p.spb), b_last = static_cast<int>((hi - 1) / p.spb);
    if (tid == 0) {
        const uint64_t start = globaltimer();
        for (int blk = b_first; blk <= b_last; ++blk) {
            int first, total;
            block_contributors(p, blk, first, total);
            const int unit = blk * p.max_slots + (total == 1 ? 0 : static_cast<int>(blockIdx.x) - first);
            while (ld_acquire_sys(p.f.tp_flags_local + unit) < static_cast<unsigned>(p.f.tp_world)) {
                if (*abort || globaltimer() - start > p.arrival_wait_ns) {
                    *abort = 1;
                    atomicExch(p.status, static_cast<unsigned>(DEV_TIMEOUT));
                    break;
                }
                __nanosleep(64);
            }
            p.f.tp_flags_local[unit] = 0u;
        }
        asm volatile("fence.acq_rel.sys;" ::: "memory");
    }
    named_bar_sync(1, CT);
    const int64_t src_stride = static_cast<int64_t>(p.M) * p.N;
    const float *recv = p.f.tp_recv[p.f.tp_rank];
    for (int blk = b_first; blk <= b_last; ++blk) {
        int first, total;
        block_contributors(p, blk, first, total);
        const int slot = total == 1 ? 0 : static_cast<int>(blockIdx.x) - first;
        const int t0 = total == 1 ? 0 : slot * TILES / total, t1 = total == 1 ? TILES : (slot + 1) * TILES / total;
        const int row0 = t0 * 16, nrows = (t1 - t0) * 16;
        const int units = ((nrows + 31) / 32) * p.M;
        constexpr int AUB = CW == 12 ? 2 : 4;  // units whose loads travel together
        for (int u0 = warp; u0 < units; u0 += CW * AUB) {
            float part[AUB][kTpMaxWorld], hpre[AUB], gpre[AUB];
#pragma unroll
            for (int k = 0; k < AUB; ++k) {
                const int u = u0 + k * CW;
                const int chunk = u / p.M, m = u - chunk * p.M;
                const int rr = chunk * 32 + lane;
                const int64_t n = static_cast<int64_t>(blk) * ROWS + row0 + rr;
                const bool ok = u < units && rr < nrows && n < p.N;
#pragma unroll
                for (int r = 0; r < kTpMaxWorld; ++r)
                    part[k][r] = (ok && r < p.f.tp_world) ? __ldcg(recv + r * src_stride + static_cast<int64_t>(m) * p.N + n)
                                                         : 0.0f;
                hpre[k] = ok ? p.f.h_out[m * p.f.ld_h_out + n] : 0.0f;
                gpre[k] = ok && p.f.next_x ? bf16_bits_to_f32(p.f.next_gamma[n]) : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < AUB; ++k) {
                const int u = u0 + k * CW;
                if (u >= units) break;  // warp-uniform
                const int chunk = u / p.M, m = u - chunk * p.M;
                const int rr = chunk * 32 + lane;
                const int64_t n = static_cast<int64_t>(blk) * ROWS + row0 + rr;
                const bool ok = rr < nrows && n < p.N;
                float v = 0.0f;
#pragma unroll
                for (int r = 0; r < kTpMaxWorld; ++r)
                    if (r < p.f.tp_world) v += part[k][r];
                resid_row(p, m, n, v, lane, ok, &hpre[k], p.f.next_x ? &gpre[k] : nullptr);
            }
        }
    }
}

// Group sums of one stage's activation columns: X_g[m] for the GPS groups
// and every activation row, via m16n8k16 MMAs with an all-ones A operand
// (rows equal, so lane (g, t) holds rows 2t, 2t+1 (+8 mt) in c[0], c[1]).
// The shared loads of GB groups are issued before their first MMA and their
// stores come last, so the MMA chains overlap instead of waiting on each
// other's stores (GB = 0: one (group, row tile) at a time, for variants
// without the registers).  Rows are written by the g == 0 lanes to
// xs[G * XSTRIDE + m].
template <int GPS, int MT, int X_BOX, int XSTRIDE, int GB>
__device__ __forceinline__ void stage_group_sums(const char *xsb, float *xs, int g, int t) {
    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};  // bf16 1.0 pairs
    if constexpr (GB == 0) {
#pragma unroll
        for (int G = 0; G < GPS; ++G)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const char *row = xsb + G * X_BOX + (g + 8 * mt) * 128;
                const uint4 v0 = *reinterpret_cast<const uint4 *>(row + (((2 * t) ^ g) << 4));
                const uint4 v1 = *reinterpret_cast<const uint4 *>(row + (((2 * t + 1) ^ g) << 4));
                float cx[4] = {0.f, 0.f, 0.f, 0.f};
                mma_bf16_16816(cx, ones, v0.x, v0.y, cx);
                mma_bf16_16816(cx, ones, v0.z, v0.w, cx);
                mma_bf16_16816(cx, ones, v1.x, v1.y, cx);
                mma_bf16_16816(cx, ones, v1.z, v1.w, cx);
                if (g == 0) {
                    xs[G * XSTRIDE + 8 * mt + 2 * t] = cx[0];
                    xs[G * XSTRIDE + 8 * mt + 2 * t + 1] = cx[1];
                }
            }
        return;
    } else {
#pragma unroll
        for (int G0 = 0; G0 < GPS; G0 += GB) {
            uint4 v[GB][MT][2];
#pragma unroll
            for (int G = 0; G < GB; ++G)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const char *row = xsb + (G0 + G) * X_BOX + (g + 8 * mt) * 128;
                    v[G][mt][0] = *reinterpret_cast<const uint4 *>(row + (((2 * t) ^ g) << 4));
                    v[G][mt][1] = *reinterpret_cast<const uint4 *>(row + (((2 * t + 1) ^ g) << 4));
                }
            float cx[GB][MT][4];
#pragma unroll
            for (int G = 0; G < GB; ++G)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    cx[G][mt][0] = cx[G][mt][1] = cx[G][mt][2] = cx[G][mt][3] = 0.f;
                    mma_bf16_16816(cx[G][mt], ones, v[G][mt][0].x, v[G][mt][0].y, cx[G][mt]);
                    mma_bf16_16816(cx[G][mt], ones, v[G][mt][0].z, v[G][mt][0].w, cx[G][mt]);
                    mma_bf16_16816(cx[G][mt], ones, v[G][mt][1].x, v[G][mt][1].y, cx[G][mt]);
                    mma_bf16_16816(cx[G][mt], ones, v[G][mt][1].z, v[G][mt][1].w, cx[G][mt]);
                }
            if (g == 0) {
#pragma unroll
                for (int G = 0; G < GB; ++G)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        xs[(G0 + G) * XSTRIDE + 8 * mt + 2 * t] = cx[G][mt][0];
                        xs[(G0 + G) * XSTRIDE + 8 * mt + 2 * t + 1] = cx[G][mt][1];
                    }
            }
        }
    }
}

// One warp's share of a stage's group sums in the warp-split kernel: groups
// part, part + T, ... (the loads of all of them first, as above).
template <int GPS, int MT, int X_BOX, int T>
__device__ __forceinline__ void stage_group_sums_part(const char *xsb, float *xs, int g, int t, int part) {
    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};  // bf16 1.0 pairs
    constexpr int NG = (GPS + T - 1) / T;
    uint4 v[NG][MT][2];
#pragma unroll
    for (int i = 0; i < NG; ++i) {
        const int G = part + i * T;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const char *row = xsb + (G < GPS ? G : 0) * X_BOX + (g + 8 * mt) * 128;
            v[i][mt][0] = *reinterpret_cast<const uint4 *>(row + (((2 * t) ^ g) << 4));
            v[i][mt][1] = *reinterpret_cast<const uint4 *>(row + (((2 * t + 1) ^ g) << 4));
        }
    }
    float cx[NG][MT][4];
#pragma unroll
    for (int i = 0; i < NG; ++i)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            cx[i][mt][0] = cx[i][mt][1] = cx[i][mt][2] = cx[i][mt][3] = 0.f;
            mma_bf16_16816(cx[i][mt], ones, v[i][mt][0].x, v[i][mt][0].y, cx[i][mt]);
            mma_bf16_16816(cx[i][mt], ones, v[i][mt][0].z, v[i][mt][0].w, cx[i][mt]);
            mma_bf16_16816(cx[i][mt], ones, v[i][mt][1].x, v[i][mt][1].y, cx[i][mt]);
            mma_bf16_16816(cx[i][mt], ones, v[i][mt][1].z, v[i][mt][1].w, cx[i][mt]);
        }
    if (g == 0) {
#pragma unroll
        for (int i = 0; i < NG; ++i) {
            const int G = part + i * T;
            if (G < GPS) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    xs[G * 16 + 8 * mt + 2 * t] = cx[i][mt][0];
                    xs[G * 16 + 8 * mt + 2 * t + 1] = cx[i][mt][1];
                }
            }
        }
    }
}

template <int BITS, int MT, int NT, int CW>
__global__ void __launch_bounds__(32 * (CW + 2), 1)
    qmv_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
               const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap xmap, Params p) {
    using Sh = Shape<BITS, MT, NT, CW>;
    constexpr int GPS = Sh::GPS, KPS = Sh::KPS, ROWS = Sh::ROWS, BOX_ROWS = Sh::BOX_ROWS;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    char *ring = smem;
    float *xsums = reinterpret_cast<float *>(ring + S * Sh::BYTES);  // [stage][group][XR]
    uint64_t *full = reinterpret_cast<uint64_t *>(xsums + MAX_STAGES * GPS * MAX_XR);
    uint64_t *empty = full + MAX_STAGES;
    uint64_t *xsfull = empty + MAX_STAGES;
    volatile int *abort = reinterpret_cast<volatile int *>(xsfull + MAX_STAGES);
    __shared__ float s_rscale[MAX_XR];  // RMSNorm row scales (row_scale mode)
    __shared__ uint64_t s_rsbar;        // completes once s_rscale holds them
    const float *rs = p.f.row_ss ? s_rscale : nullptr;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The next kernel may launch once every CTA of this grid has started.
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW + 1);  // consumer warps and the sum warp
            mbar_init(&xsfull[s], 1);
        }
        mbar_init(&s_rsbar, 1);
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const int64_t T = p.items;
    const int64_t lo = static_cast<int64_t>(blockIdx.x) * T / gridDim.x;
    const int64_t hi = static_cast<int64_t>(blockIdx.x + 1) * T / gridDim.x;
    const int g = lane >> 2, t = lane & 3;

    if (warp == CW) {  // ------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            tma_prefetch_desc(&smap);
            tma_prefetch_desc(&bmap);
            tma_prefetch_desc(&xmap);
            const uint64_t stream_policy = l2_evict_first();
            auto load_params = [&](int stage, int64_t i) {
                const int blk = static_cast<int>(i / p.spb), st = static_cast<int>(i - int64_t(blk) * p.spb);
                char *dst = ring + stage * Sh::BYTES;
                mbar_arrive_expect_tx(&full[stage], Sh::TX_BYTES);
                const int kk = st * KPS;
                const int g8 = (kk / GROUP) & ~7;
#pragma unroll
                for (int bx = 0; bx < ROWS / BOX_ROWS; ++bx) {
                    const int row0 = blk * ROWS + bx * BOX_ROWS;
                    tma_load_2d_hint(dst + bx * BOX_ROWS * 128, &wmap, &full[stage], kk * BITS / 32, row0, stream_policy);
                    tma_load_2d_hint(dst + Sh::W + bx * BOX_ROWS * 16, &smap, &full[stage], g8, row0, stream_policy);
                    tma_load_2d_hint(dst + Sh::W + Sh::SB + bx * BOX_ROWS * 16, &bmap, &full[stage], g8, row0,
                                     stream_policy);
                }
            };
            auto load_x = [&](int stage, int64_t i) {  // box: 64 columns x XR rows x GPS groups
                const int blk = static_cast<int>(i / p.spb), st = static_cast<int>(i - int64_t(blk) * p.spb);
                tma_load_3d(ring + stage * Sh::BYTES + Sh::W + 2 * Sh::SB, &xmap, &full[stage], 0, 0, st * GPS);
            };
            // First pass over the ring: weights, scales and biases need nothing
            // from the preceding kernel; the activations do.
            const int pre = static_cast<int>(min(hi - lo, static_cast<int64_t>(S)));
            for (int j = 0; j < pre; ++j) load_params(j, lo + j);
            pdl_wait();
            for (int j = 0; j < pre; ++j) load_x(j, lo + j);
            int stage = pre % S;
            uint32_t phase = pre == S ? 1u : 0u;
            uint32_t issued_mask = (1u << pre) - 1u, issued_par = 0;  // stages 0..pre-1 at parity 0
            for (int64_t i = lo + pre; i < hi; ++i) {
                // On a timed-out wait (abort set) stop issuing loads; the other
                // roles walk to the end without waiting.  A stage is never
                // re-armed after an abort: a stage whose loads did not all
                // land has an unfinished phase.
                if (!mbar_wait(&empty[stage], phase ^ 1, abort, p.status) || *abort) break;
                load_params(stage, i);
                load_x(stage, i);
                issued_mask |= 1u << stage;
                issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                if (++stage == S) { stage = 0; phase ^= 1; }
            }
            // Let every copy this CTA issued land before the CTA exits.
            for (int s = 0; s < S; ++s)
                if (issued_mask & (1u << s)) mbar_wait_drain(&full[s], (issued_par >> s) & 1u);
        }
        __syncwarp();
    } else if (warp == CW + 1) {  // ----------------------------- group sums
        pdl_wait();
        // Row scales rsqrt(sum_k h^2 / K + eps) of the unnormalised
        // activations from their per-16-column sums of squares: lane l adds
        // tiles l, l + 32, ... for every row, then a butterfly per row -- the
        // RMSNorm prologue's order.  Only the epilogues use them, so their
        // loads ride along the stage loop: each stage issues the next two
        // tiles per lane before waiting for its data and adds them after its
        // group sums, and the scales are published through s_rsbar.
        constexpr int RMAX = 8 * MT, RQ = RMAX / 4;  // activation rows this instantiation serves
        const int quads = (p.M + 3) / 4;
        float racc[RMAX];
#pragma unroll
        for (int m = 0; m < RMAX; ++m) racc[m] = 0.0f;
        float4 rv[2][RQ];
        int rs_left = p.f.row_ss ? max(1, (p.f.ss_tiles + 63) / 64) : 0, rtile = lane;
        auto rs_issue = [&]() {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int tl = rtile + 32 * j;
                const float4 *row = reinterpret_cast<const float4 *>(p.f.row_ss + tl * kSsWidth);
#pragma unroll
                for (int q = 0; q < RQ; ++q)
                    rv[j][q] = (tl < p.f.ss_tiles && q < quads) ? __ldcg(row + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        auto rs_accum = [&]() {
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int q = 0; q < RQ; ++q) {
                    racc[4 * q] += rv[j][q].x;
                    racc[4 * q + 1] += rv[j][q].y;
                    racc[4 * q + 2] += rv[j][q].z;
                    racc[4 * q + 3] += rv[j][q].w;
                }
            rtile += 64;
            if (--rs_left == 0) {
                // Butterfly of every row (levels outermost, so the rows'
                // shuffle chains overlap), then lane m forms row m's scale.
#pragma unroll
                for (int o = 16; o; o >>= 1)
#pragma unroll
                    for (int m = 0; m < RMAX; ++m) racc[m] += __shfl_xor_sync(0xffffffffu, racc[m], o);
                float mine = 0.0f;
#pragma unroll
                for (int m = 0; m < RMAX; ++m) mine = lane == m ? racc[m] : mine;
                if (lane < RMAX && lane < p.M) s_rscale[lane] = rsqrtf(mine / static_cast<float>(p.K) + p.f.eps);
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_rsbar);
            }
        };
        // X_g = sum_{k in g} x[m][k] for every activation row, once per CTA and
        // stage (stage_group_sums).
        int stage = 0;
        uint32_t phase = 0;
        for (int64_t i = lo; i < hi; ++i) {
            const bool rs_step = rs_left > 0;
            if (rs_step) rs_issue();
            mbar_wait(&full[stage], phase, abort, p.status);
            const char *xsb = ring + stage * Sh::BYTES + Sh::W + 2 * Sh::SB;
            stage_group_sums<GPS, MT, Sh::X_BOX, MAX_XR, (MT > 2 ? 0 : CW >= 12 ? 1 : GPS)>(
                xsb, xsums + stage * GPS * MAX_XR, g, t);
            fence_proxy_async_smem();  // x reads before the stage's next TMA fill
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&xsfull[stage]);
                mbar_arrive(&empty[stage]);
            }
            if (rs_step) rs_accum();
            if (++stage == S) { stage = 0; phase ^= 1; }
        }
        while (rs_left > 0) {  // a range shorter than the tiles' loads
            rs_issue();
            rs_accum();
        }
    } else {  // ------------------------------------------------- consumers
        pdl_wait();
        int stage = 0;
        uint32_t phase = 0;
        int64_t i = lo;
        while (i < hi) {
            const int blk = static_cast<int>(i / p.spb);
            const int64_t blk_begin = static_cast<int64_t>(blk) * p.spb;
            const int64_t seg_end = min(hi, blk_begin + p.spb);
            uint64_t acc[NT][MT][2];  // packed f32 pairs: [..][0] = (c0, c1), [..][1] = (c2, c3)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) acc[nt][mt][0] = acc[nt][mt][1] = 0ull;

            for (; i < seg_end; ++i) {
                const int j = static_cast<int>(i - blk_begin);  // stage index within the block
                // A timed-out wait sets *abort; keep walking the loop (results are
                // then garbage and the status word says TIMEOUT) so that every
                // consumer reaches the same barriers and no thread hangs.
                mbar_wait(&full[stage], phase, abort, p.status);
                const char *sw = ring + stage * Sh::BYTES;
                const char *ssb = sw + Sh::W;
                const char *bsb = ssb + Sh::SB;
                const char *xsb = bsb + Sh::SB;
                const int go0 = (j * GPS) & 7;  // first group of this stage within the 8-group scale box
                uint32_t sv[NT][2][GPS / 2], bv[NT][2][GPS / 2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int r = (warp * NT + nt) * 16 + g + 8 * h;
                        if constexpr (GPS == 4) {
                            const uint2 a2 = *reinterpret_cast<const uint2 *>(ssb + r * 16 + go0 * 2);
                            const uint2 b2 = *reinterpret_cast<const uint2 *>(bsb + r * 16 + go0 * 2);
                            sv[nt][h][0] = a2.x; sv[nt][h][1] = a2.y; bv[nt][h][0] = b2.x; bv[nt][h][1] = b2.y;
                        } else {
                            sv[nt][h][0] = *reinterpret_cast<const uint32_t *>(ssb + r * 16 + go0 * 2);
                            bv[nt][h][0] = *reinterpret_cast<const uint32_t *>(bsb + r * 16 + go0 * 2);
                        }
                    }
                mbar_wait(&xsfull[stage], phase, abort, p.status);
                const float *xs = xsums + stage * GPS * MAX_XR;
#pragma unroll
                for (int G = 0; G < GPS; ++G) {
                    // B fragments: row m = g + 8*mt of the group's XR x 64 box,
                    // columns 16t..16t+15 = 16-byte chunks 2t, 2t+1 stored at
                    // chunk ^ (m % 8) (128-byte swizzle).
                    uint32_t xf[MT][8];
                    const char *xb = xsb + G * Sh::X_BOX;
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const char *row = xb + (g + 8 * mt) * 128;
                        const uint4 v0 = *reinterpret_cast<const uint4 *>(row + (((2 * t) ^ g) << 4));
                        const uint4 v1 = *reinterpret_cast<const uint4 *>(row + (((2 * t + 1) ^ g) << 4));
                        xf[mt][0] = v0.x; xf[mt][1] = v0.y; xf[mt][2] = v0.z; xf[mt][3] = v0.w;
                        xf[mt][4] = v1.x; xf[mt][5] = v1.y; xf[mt][6] = v1.z; xf[mt][7] = v1.w;
                    }
                    // A fragments of the warp's tiles and all four k-steps first,
                    // then the MMAs with tiles and m-tiles interleaved (NT * MT
                    // independent accumulator chains).
                    uint32_t a[NT][4][4];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const char *tw = sw + ((warp * NT + nt) * 16 + g) * 128;  // rows r and r + 8
                        if constexpr (BITS == 4) {
                            const int off = (((2 * G + (t >> 1)) ^ g) << 4) + (t & 1) * 8;
                            const uint2 u0 = *reinterpret_cast<const uint2 *>(tw + off);
                            const uint2 u1 = *reinterpret_cast<const uint2 *>(tw + 8 * 128 + off);
                            const uint32_t w0[2] = {u0.x, u0.y}, w1[2] = {u1.x, u1.y};
#pragma unroll
                            for (int s = 0; s < 4; ++s) {
                                const int p0 = 2 * (s & 1);
                                a[nt][s][0] = dec4(w0[s >> 1], p0);
                                a[nt][s][1] = dec4(w1[s >> 1], p0);
                                a[nt][s][2] = dec4(w0[s >> 1], p0 + 1);
                                a[nt][s][3] = dec4(w1[s >> 1], p0 + 1);
                            }
                        } else {
                            const int off = ((4 * G + t) ^ g) << 4;
                            const uint4 u0 = *reinterpret_cast<const uint4 *>(tw + off);
                            const uint4 u1 = *reinterpret_cast<const uint4 *>(tw + 8 * 128 + off);
                            const uint32_t w0[4] = {u0.x, u0.y, u0.z, u0.w}, w1[4] = {u1.x, u1.y, u1.z, u1.w};
#pragma unroll
                            for (int s = 0; s < 4; ++s) {
                                a[nt][s][0] = dec8(w0[s], 0);
                                a[nt][s][1] = dec8(w1[s], 0);
                                a[nt][s][2] = dec8(w0[s], 2);
                                a[nt][s][3] = dec8(w1[s], 2);
                            }
                        }
                    }
                    float c[NT][MT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) c[nt][mt][0] = c[nt][mt][1] = c[nt][mt][2] = c[nt][mt][3] = 0.f;
#pragma unroll
                    for (int s = 0; s < 4; ++s)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                const uint32_t b0 = BITS == 4 ? xf[mt][4 * (s >> 1) + 2 * (s & 1)] : xf[mt][2 * s];
                                const uint32_t b1 =
                                    BITS == 4 ? xf[mt][4 * (s >> 1) + 2 * (s & 1) + 1] : xf[mt][2 * s + 1];
                                mma_bf16_16816(c[nt][mt], a[nt][s], b0, b1, c[nt][mt]);
                            }
                    uint64_t xsum[MT];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        xsum[mt] = *reinterpret_cast<const uint64_t *>(xs + G * MAX_XR + 8 * mt + 2 * t);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const uint32_t s_w0 = sv[nt][0][G >> 1], s_w1 = sv[nt][1][G >> 1];
                        const uint32_t b_w0 = bv[nt][0][G >> 1], b_w1 = bv[nt][1][G >> 1];
                        const float s0 = __uint_as_float((G & 1) ? (s_w0 & 0xFFFF0000u) : (s_w0 << 16));
                        const float s1 = __uint_as_float((G & 1) ? (s_w1 & 0xFFFF0000u) : (s_w1 << 16));
                        float q0 = __uint_as_float((G & 1) ? (b_w0 & 0xFFFF0000u) : (b_w0 << 16));
                        float q1 = __uint_as_float((G & 1) ? (b_w1 & 0xFFFF0000u) : (b_w1 << 16));
                        if constexpr (BITS == 4) {  // codes entered the MMA as 128+q
                            q0 = fmaf(-128.0f, s0, q0);
                            q1 = fmaf(-128.0f, s1, q1);
                        }
                        const uint64_t s0p = f2_pack(s0, s0), s1p = f2_pack(s1, s1);
                        const uint64_t q0p = f2_pack(q0, q0), q1p = f2_pack(q1, q1);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            acc[nt][mt][0] = fma_f32x2(s0p, f2_pack(c[nt][mt][0], c[nt][mt][1]),
                                                       fma_f32x2(q0p, xsum[mt], acc[nt][mt][0]));
                            acc[nt][mt][1] = fma_f32x2(s1p, f2_pack(c[nt][mt][2], c[nt][mt][3]),
                                                       fma_f32x2(q1p, xsum[mt], acc[nt][mt][1]));
                        }
                    }
                }
                // The stage is refilled by TMA (async proxy) after this release;
                // order this warp's generic-proxy reads of it first.
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[stage]);
                if (++stage == S) { stage = 0; phase ^= 1; }
            }
            float accf[NT][MT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    accf[nt][mt][0] = __uint_as_float(static_cast<uint32_t>(acc[nt][mt][0]));
                    accf[nt][mt][1] = __uint_as_float(static_cast<uint32_t>(acc[nt][mt][0] >> 32));
                    accf[nt][mt][2] = __uint_as_float(static_cast<uint32_t>(acc[nt][mt][1]));
                    accf[nt][mt][3] = __uint_as_float(static_cast<uint32_t>(acc[nt][mt][1] >> 32));
                }
            segment_epilogue<MT, NT, CW>(p, accf, blk, warp, g, t, tid, rs, &s_rsbar, abort);
        }
        combine_blocks<ROWS, CW>(p, lo, hi, warp, lane, tid, abort, rs, &s_rsbar);
        if (p.f.epi == EPI_RESID_AR) ar_finish<ROWS, CW>(p, lo, hi, warp, lane, tid, abort);
    }
}

// Warp-split whole-K kernel (M <= 16, N up to three 16-row tiles per SM).
// One block of T 16-row tiles per CTA, streamed over the whole K range once,
// so no block is combined across CTAs: consumer warp (tile t, K lane k of
// KW) takes stages k, k + KW, k + 2 KW, ... of tile t.  The group sums X_g
// of a stage (the stream-K kernel's all-ones MMAs, same order) are split
// over the T warps of its K lane -- warp t forms groups t, t + T, ... into a
// small shared ring beside the stage ring -- and the lane's warps meet on a
// named barrier before using them, so the affine per-group step is the
// stream-K kernel's.  The K lanes' accumulators meet in
// shared memory and are added in lane order (results do not depend on
// scheduling); the lane-0 warps apply the epilogue.  The ring depth is a
// multiple of KW, so every ring slot serves the stages of one K lane only: a
// warp waiting on a slot has consumed the slot's previous stage itself, and
// its parity wait never runs a phase ahead.  A stage is two TMA loads (the
// packed rows; the activation columns of its groups as one 3D box), the
// block's scales and biases one load each per launch: at these block heights
// the TMA work per stage, not its bytes, sets the streaming rate.  The spare
// warp fetches what the epilogue reads (the residual rows and next-norm
// weights) into shared memory at the start, while the stages stream, and
// forms the RMSNorm row scales.  A lane's group-sum slot is rewritten only
// after its warps met on a later stage's barrier, so the ring depth is at
// least 2 KW.
template <int BITS, int MT, int T>
struct WsShape {
    static constexpr int KW = T == 3 ? 3 : 10 / T;  // K lanes
    static constexpr int CW = T * KW;               // consumer warps
    static constexpr int THREADS = 32 * (CW + 2);   // consumers, producer, spare warp
    static constexpr int ROWS = 16 * T;
    static constexpr int XR = 16;
    static constexpr int X_BOX = XR * 128;
    static constexpr int GPS = BITS == 4 ? 4 : 2;
    static constexpr int KPS = GPS * GROUP;
    static constexpr int W = ROWS * 128;
    static constexpr int X = GPS * X_BOX;
    static constexpr int BYTES = W + X;     // a ring stage: packed rows, then the activation columns
    static constexpr int TX_BYTES = W + X;  // bytes the stage's two TMA loads deliver
    static constexpr int RED = KW * T * MT * 4 * 32 * 4;  // the K lanes' accumulators
    static_assert(W % 1024 == 0 && X % 1024 == 0 && RED % 16 == 0, "stage layout");
};

// Scales and biases of a warp-split block live in shared memory for the
// whole launch (one load each): [ROWS][pitch] bf16, the pitch the group count
// rounded up to 16 plus 8, so the eight rows a warp reads at once fall in
// distinct banks (pitch/2 words = 4 mod 8).  The padding columns are read
// beyond the tensor's extent and come back zero.
__host__ __device__ constexpr int ws_slab_pitch(int K) { return (K / GROUP + 15) / 16 * 16 + 8; }
__host__ __device__ constexpr int ws_slab_bytes(int rows, int K) { return (2 * rows * ws_slab_pitch(K) * 2 + 127) / 128 * 128; }

static_assert(WsShape<4, 2, 1>::ROWS == kVariantBoxRows[6] && WsShape<4, 2, 2>::ROWS == kVariantBoxRows[7] &&
                  WsShape<4, 2, 3>::ROWS == kVariantBoxRows[8],
              "tensor-map boxes match the warp-split kernels' blocks");

// Row scales of the RMSNorm prologue, one warp: lane l adds tiles l, l + 32,
// ... (four tiles' loads in flight per round), then a butterfly per row --
// the same order as the stream-K kernel and the prep kernel.
template <int MT>
__device__ void ws_row_scales(const Params &p, int lane, float *s_rscale, uint64_t *bar) {
    constexpr int RMAX = 8 * MT, RQ = RMAX / 4, TPR = 4;
    const int quads = (p.M + 3) / 4;
    float racc[RMAX];
#pragma unroll
    for (int m = 0; m < RMAX; ++m) racc[m] = 0.0f;
    for (int tl0 = lane; tl0 < p.f.ss_tiles; tl0 += 32 * TPR) {
        float4 v[TPR][RQ];
#pragma unroll
        for (int j = 0; j < TPR; ++j) {
            const int tl = tl0 + 32 * j;
            const float4 *row = reinterpret_cast<const float4 *>(p.f.row_ss + tl * kSsWidth);
#pragma unroll
            for (int q = 0; q < RQ; ++q)
                v[j][q] = (tl < p.f.ss_tiles && q < quads) ? __ldcg(row + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < TPR; ++j)
#pragma unroll
            for (int q = 0; q < RQ; ++q) {
                racc[4 * q] += v[j][q].x;
                racc[4 * q + 1] += v[j][q].y;
                racc[4 * q + 2] += v[j][q].z;
                racc[4 * q + 3] += v[j][q].w;
            }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int m = 0; m < RMAX; ++m) racc[m] += __shfl_xor_sync(0xffffffffu, racc[m], o);
    float mine = 0.0f;
#pragma unroll
    for (int m = 0; m < RMAX; ++m) mine = lane == m ? racc[m] : mine;
    if (lane < RMAX && lane < p.M) s_rscale[lane] = rsqrtf(mine / static_cast<float>(p.K) + p.f.eps);
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

template <int BITS, int MT, int T>
__global__ void __launch_bounds__(WsShape<BITS, MT, T>::THREADS, 1)
    qmv_ws_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                  const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap xmap, Params p) {
    using Sh = WsShape<BITS, MT, T>;
    constexpr int GPS = Sh::GPS, KPS = Sh::KPS, KW = Sh::KW, CW = Sh::CW, ROWS = Sh::ROWS;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;  // a multiple of KW
    const int SP = ws_slab_pitch(p.K);
    char *ring = smem;
    char *slab = ring + S * Sh::BYTES;  // scales [ROWS][SP], then biases [ROWS][SP]
    float *red = reinterpret_cast<float *>(slab + ws_slab_bytes(ROWS, p.K));
    float *xsums = red + Sh::RED / 4;               // [slot][group][16 activation rows]
    float *hg = xsums + MAX_WS_STAGES * GPS * 16;    // residual operands [tile][mt][h][4][lane]
    uint64_t *full = reinterpret_cast<uint64_t *>(hg + T * MT * 8 * 32);
    uint64_t *empty = full + MAX_WS_STAGES;
    uint64_t *sbfull = empty + MAX_WS_STAGES;
    uint64_t *hgbar = sbfull + 1;
    volatile int *abort = reinterpret_cast<volatile int *>(hgbar + 1);
    __shared__ float s_rscale[MAX_XR];  // RMSNorm row scales (row_scale mode)
    __shared__ uint64_t s_rsbar;        // completes once s_rscale holds them
    const float *rs = p.f.row_ss ? s_rscale : nullptr;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], T);  // the T warps of the slot's K lane
        }
        mbar_init(sbfull, 1);
        mbar_init(hgbar, 1);
        mbar_init(&s_rsbar, 1);
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int blk = blockIdx.x, spb = p.spb;
    const int g = lane >> 2, t = lane & 3;

    if (warp == CW) {  // ------------------------------------------ producer
        const uint64_t stream_policy = l2_evict_first();
        const int row0 = blk * ROWS, pre = min(spb, S);
        auto load_params = [&](int slot, int j) {
            mbar_arrive_expect_tx(&full[slot], Sh::TX_BYTES);
            tma_load_2d_hint(ring + slot * Sh::BYTES, &wmap, &full[slot], j * KPS * BITS / 32, row0, stream_policy);
        };
        auto load_x = [&](int slot, int j) {  // box: 64 columns x 16 rows x GPS groups
            tma_load_3d(ring + slot * Sh::BYTES + Sh::W, &xmap, &full[slot], 0, 0, j * GPS);
        };
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            tma_prefetch_desc(&smap);
            tma_prefetch_desc(&bmap);
            tma_prefetch_desc(&xmap);
            // The block's scales and biases (box: SP groups x ROWS rows).
            mbar_arrive_expect_tx(sbfull, 2 * ROWS * SP * 2);
            tma_load_2d_hint(slab, &smap, sbfull, 0, row0, stream_policy);
            tma_load_2d_hint(slab + ROWS * SP * 2, &bmap, sbfull, 0, row0, stream_policy);
            // Weights of the first ring fill need nothing from the preceding
            // kernel; the activations do.
            for (int j = 0; j < pre; ++j) load_params(j, j);
            pdl_wait();
            for (int j = 0; j < pre; ++j) load_x(j, j);
        }
        if (lane == 0) {
            uint32_t issued_mask = pre >= 32 ? ~0u : (1u << pre) - 1u, issued_par = 0;
            for (int j = pre; j < spb; ++j) {
                const int slot = j % S;
                const uint32_t ph = static_cast<uint32_t>(j / S) & 1u;
                // Never re-arm a slot after an abort (see the stream-K producer).
                if (!mbar_wait(&empty[slot], ph ^ 1u, abort, p.status) || *abort) break;
                load_params(slot, j);
                load_x(slot, j);
                issued_mask |= 1u << slot;
                issued_par = (issued_par & ~(1u << slot)) | (ph << slot);
            }
            for (int s = 0; s < S; ++s)
                if (issued_mask & (1u << s)) mbar_wait_drain(&full[s], (issued_par >> s) & 1u);
            mbar_wait_drain(sbfull, 0);
        }
        __syncwarp();
    } else if (warp == CW + 1) {  // --------- epilogue operands, row scales
        pdl_wait();
        if (p.f.epi == EPI_RESID) {
            for (int tl = 0; tl < T; ++tl) {
                float pre[MT][2][4];
                load_resid_operands<MT>(p, static_cast<int64_t>(blk) * ROWS + tl * 16, g, t, pre);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int e = 0; e < 4; ++e) hg[(((tl * MT + mt) * 2 + h) * 4 + e) * 32 + lane] = pre[mt][h][e];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(hgbar);
        }
        if (rs) ws_row_scales<MT>(p, lane, s_rscale, &s_rsbar);
    } else {  // ------------------------------------------------- consumers
        pdl_wait();
        const int tile = warp % T, kl = warp / T;
        uint64_t acc[MT][2];  // packed f32 pairs: [..][0] = (c0, c1), [..][1] = (c2, c3)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = 0ull;
        if (kl < spb) mbar_wait(sbfull, 0, abort, p.status);
        const char *ssl = slab + (tile * 16 + g) * SP * 2, *bsl = ssl + ROWS * SP * 2;  // row r; row r + 8 at +8 SP
        for (int j = kl; j < spb; j += KW) {
            const int slot = j % S;
            const uint32_t ph = static_cast<uint32_t>(j / S) & 1u;
            mbar_wait(&full[slot], ph, abort, p.status);
            const char *sw = ring + slot * Sh::BYTES;
            const char *xsb = sw + Sh::W;
            float *xs = xsums + slot * GPS * 16;
            uint32_t sv[2][GPS / 2], bv[2][GPS / 2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int off = h * 8 * SP * 2 + j * GPS * 2;  // groups j*GPS .. j*GPS+GPS-1
                if constexpr (GPS == 4) {
                    const uint2 a2 = *reinterpret_cast<const uint2 *>(ssl + off);
                    const uint2 b2 = *reinterpret_cast<const uint2 *>(bsl + off);
                    sv[h][0] = a2.x; sv[h][1] = a2.y; bv[h][0] = b2.x; bv[h][1] = b2.y;
                } else {
                    sv[h][0] = *reinterpret_cast<const uint32_t *>(ssl + off);
                    bv[h][0] = *reinterpret_cast<const uint32_t *>(bsl + off);
                }
            }
            // This warp's share of the stage's group sums, then the K lane's
            // warps meet (named barrier 2 + k).
            stage_group_sums_part<GPS, MT, Sh::X_BOX, T>(xsb, xs, g, t, tile);
            if constexpr (T > 1) named_bar_sync(2 + kl, T * 32);
#pragma unroll
            for (int G = 0; G < GPS; ++G) {
                uint32_t xf[MT][8];
                const char *xb = xsb + G * Sh::X_BOX;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const char *row = xb + (g + 8 * mt) * 128;
                    const uint4 v0 = *reinterpret_cast<const uint4 *>(row + (((2 * t) ^ g) << 4));
                    const uint4 v1 = *reinterpret_cast<const uint4 *>(row + (((2 * t + 1) ^ g) << 4));
                    xf[mt][0] = v0.x; xf[mt][1] = v0.y; xf[mt][2] = v0.z; xf[mt][3] = v0.w;
                    xf[mt][4] = v1.x; xf[mt][5] = v1.y; xf[mt][6] = v1.z; xf[mt][7] = v1.w;
                }
                uint32_t a[4][4];
                const char *tw = sw + (tile * 16 + g) * 128;  // rows r and r + 8
                if constexpr (BITS == 4) {
                    const int off = (((2 * G + (t >> 1)) ^ g) << 4) + (t & 1) * 8;
                    const uint2 u0 = *reinterpret_cast<const uint2 *>(tw + off);
                    const uint2 u1 = *reinterpret_cast<const uint2 *>(tw + 8 * 128 + off);
                    const uint32_t w0[2] = {u0.x, u0.y}, w1[2] = {u1.x, u1.y};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const int p0 = 2 * (s & 1);
                        a[s][0] = dec4(w0[s >> 1], p0);
                        a[s][1] = dec4(w1[s >> 1], p0);
                        a[s][2] = dec4(w0[s >> 1], p0 + 1);
                        a[s][3] = dec4(w1[s >> 1], p0 + 1);
                    }
                } else {
                    const int off = ((4 * G + t) ^ g) << 4;
                    const uint4 u0 = *reinterpret_cast<const uint4 *>(tw + off);
                    const uint4 u1 = *reinterpret_cast<const uint4 *>(tw + 8 * 128 + off);
                    const uint32_t w0[4] = {u0.x, u0.y, u0.z, u0.w}, w1[4] = {u1.x, u1.y, u1.z, u1.w};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        a[s][0] = dec8(w0[s], 0);
                        a[s][1] = dec8(w1[s], 0);
                        a[s][2] = dec8(w0[s], 2);
                        a[s][3] = dec8(w1[s], 2);
                    }
                }
                float c[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) c[mt][i] = 0.f;
#pragma unroll
                for (int s = 0; s < 4; ++s)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint32_t b0 = BITS == 4 ? xf[mt][4 * (s >> 1) + 2 * (s & 1)] : xf[mt][2 * s];
                        const uint32_t b1 = BITS == 4 ? xf[mt][4 * (s >> 1) + 2 * (s & 1) + 1] : xf[mt][2 * s + 1];
                        mma_bf16_16816(c[mt], a[s], b0, b1, c[mt]);
                    }
                const uint32_t s_w0 = sv[0][G >> 1], s_w1 = sv[1][G >> 1];
                const uint32_t b_w0 = bv[0][G >> 1], b_w1 = bv[1][G >> 1];
                const float s0 = __uint_as_float((G & 1) ? (s_w0 & 0xFFFF0000u) : (s_w0 << 16));
                const float s1 = __uint_as_float((G & 1) ? (s_w1 & 0xFFFF0000u) : (s_w1 << 16));
                float q0 = __uint_as_float((G & 1) ? (b_w0 & 0xFFFF0000u) : (b_w0 << 16));
                float q1 = __uint_as_float((G & 1) ? (b_w1 & 0xFFFF0000u) : (b_w1 << 16));
                if constexpr (BITS == 4) {  // codes entered the MMA as 128+q
                    q0 = fmaf(-128.0f, s0, q0);
                    q1 = fmaf(-128.0f, s1, q1);
                }
                const uint64_t s0p = f2_pack(s0, s0), s1p = f2_pack(s1, s1);
                const uint64_t q0p = f2_pack(q0, q0), q1p = f2_pack(q1, q1);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint64_t xsum = *reinterpret_cast<const uint64_t *>(xs + G * 16 + 8 * mt + 2 * t);
                    acc[mt][0] = fma_f32x2(s0p, f2_pack(c[mt][0], c[mt][1]), fma_f32x2(q0p, xsum, acc[mt][0]));
                    acc[mt][1] = fma_f32x2(s1p, f2_pack(c[mt][2], c[mt][3]), fma_f32x2(q1p, xsum, acc[mt][1]));
                }
            }
            // The slot is refilled by TMA (async proxy) after this release;
            // order this warp's generic-proxy reads of it first.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        float accf[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            accf[mt][0] = __uint_as_float(static_cast<uint32_t>(acc[mt][0]));
            accf[mt][1] = __uint_as_float(static_cast<uint32_t>(acc[mt][0] >> 32));
            accf[mt][2] = __uint_as_float(static_cast<uint32_t>(acc[mt][1]));
            accf[mt][3] = __uint_as_float(static_cast<uint32_t>(acc[mt][1] >> 32));
        }
        // K lanes 1..KW-1 hand their sums to lane 0 of their tile, which adds
        // them in lane order.  red[((k * T + tile) * MT + mt) * 4 + i][lane].
        if (kl > 0) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) red[(((kl * T + tile) * MT + mt) * 4 + i) * 32 + lane] = accf[mt][i];
        }
        named_bar_sync(1, CW * 32);
        if (kl == 0) {
            for (int k = 1; k < KW; ++k)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) accf[mt][i] += red[(((k * T + tile) * MT + mt) * 4 + i) * 32 + lane];
            if (rs) mbar_wait(&s_rsbar, 0, abort, p.status);  // the row scales are out
            const int64_t n0 = static_cast<int64_t>(blk) * ROWS + tile * 16;
            if (p.f.epi == EPI_RESID) {
                mbar_wait(hgbar, 0, abort, p.status);
                float pre[MT][2][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int e = 0; e < 4; ++e) pre[mt][h][e] = hg[(((tile * MT + mt) * 2 + h) * 4 + e) * 32 + lane];
                finish_tile<MT>(p, accf, n0, g, t, rs, pre);
            } else {
                finish_tile<MT>(p, accf, n0, g, t, rs);
            }
        }
        if (p.f.epi == EPI_RESID_AR) {
            ar_signal<CW>(p, blk * p.max_slots, tid);
            ar_finish<ROWS, CW>(p, static_cast<int64_t>(blk) * spb, static_cast<int64_t>(blk + 1) * spb, warp, lane,
                                tid, abort);
        }
    }
}

// Activations into the kernel's layout: dst[m][k] = bf16(src) in pair order
// (4-bit) or natural order (8-bit).  mode 0: src is bf16 x; mode 1: src is
// rmsnorm of the f32 residual stream h with the per-16-column sums of squares
// `ss` ([ss_tiles][16]) and weights gamma.
__global__ void prep_kernel(const void *src, int64_t ld_src, int mode, const float *ss, int ss_tiles,
                            const uint16_t *gamma, float eps, int M, int K, int pair_order, uint16_t *dst,
                            int64_t ld_dst) {
    __shared__ float rms[kMaxQmvRows];
    pdl_wait();
    if (mode == 1) {
        // 1/rms per row: one warp per row, fixed summation order.
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int m = w; m < M; m += blockDim.x / 32) {
            float sum = 0.0f;
            for (int tl = lane; tl < ss_tiles; tl += 32) sum += ss[tl * kSsWidth + m];
#pragma unroll
            for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) rms[m] = rsqrtf(sum / static_cast<float>(K) + eps);
        }
        __syncthreads();
    }
    const int64_t words = static_cast<int64_t>(M) * (K / 8);
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < words;
         c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int m = static_cast<int>(c / (K / 8));
        const int k0 = static_cast<int>(c % (K / 8)) * 8;
        uint32_t v[4];
        if (mode == 1) {
            const float4 *hp = reinterpret_cast<const float4 *>(static_cast<const float *>(src) + m * ld_src + k0);
            const float4 h0 = hp[0], h1 = hp[1];
            const uint4 gm = *reinterpret_cast<const uint4 *>(gamma + k0);
            const float hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            const uint32_t gw[4] = {gm.x, gm.y, gm.z, gm.w};
            const float r = rms[m];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t lo = f32_to_bf16_bits(hv[2 * e] * r * __uint_as_float(gw[e] << 16));
                const uint32_t hi = f32_to_bf16_bits(hv[2 * e + 1] * r * __uint_as_float(gw[e] & 0xFFFF0000u));
                v[e] = lo | (hi << 16);
            }
        } else {
            const uint4 u = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(src) + m * ld_src + k0);
            v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
        }
        uint4 o;
        if (pair_order) {  // [x0 x4 x1 x5 x2 x6 x3 x7]
            o.x = prmt(v[0], v[2], 0x5410u);
            o.y = prmt(v[0], v[2], 0x7632u);
            o.z = prmt(v[1], v[3], 0x5410u);
            o.w = prmt(v[1], v[3], 0x7632u);
        } else {
            o = make_uint4(v[0], v[1], v[2], v[3]);
        }
        *reinterpret_cast<uint4 *>(dst + m * ld_dst + k0) = o;
    }
}

// Residual add and RMSNorm for the tensor-parallel decoder: one CTA per
// activation row m.  h[m] += add[m] (when add is given; f32, in place), then
// dst[m] = bf16(h[m] * rsqrt(mean(h[m]^2) + eps) * gamma) in the qmv's column
// order.  The sum of squares is formed in a fixed order (per-thread partial
// sums over a fixed column assignment, then a fixed tree), so every rank that
// holds the same h computes the same bits.
template <int PER>
__global__ void __launch_bounds__(256) resid_norm_kernel(float *h, int64_t ld_h, const float *add, int64_t ld_add,
                                                         const uint16_t *gamma, float eps, int K, int pair_order,
                                                         uint16_t *dst, int64_t ld_dst) {
    __shared__ float red[8];
    pdl_wait();
    const int m = blockIdx.x, tid = threadIdx.x;
    float *hr = h + static_cast<int64_t>(m) * ld_h;
    const float *ar = add ? add + static_cast<int64_t>(m) * ld_add : nullptr;
    float v[PER * 8];
    float ssq = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int k0 = (j * 256 + tid) * 8;
        if (k0 < K) {
            float4 a0 = *reinterpret_cast<const float4 *>(hr + k0), a1 = *reinterpret_cast<const float4 *>(hr + k0 + 4);
            if (ar) {
                const float4 b0 = *reinterpret_cast<const float4 *>(ar + k0);
                const float4 b1 = *reinterpret_cast<const float4 *>(ar + k0 + 4);
                a0.x += b0.x; a0.y += b0.y; a0.z += b0.z; a0.w += b0.w;
                a1.x += b1.x; a1.y += b1.y; a1.z += b1.z; a1.w += b1.w;
                *reinterpret_cast<float4 *>(hr + k0) = a0;
                *reinterpret_cast<float4 *>(hr + k0 + 4) = a1;
            }
            const float e[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[j * 8 + i] = e[i];
                ssq = fmaf(e[i], e[i], ssq);
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
    if ((tid & 31) == 0) red[tid >> 5] = ssq;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float r = rsqrtf(tot / static_cast<float>(K) + eps);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int k0 = (j * 256 + tid) * 8;
        if (k0 < K) {
            const uint4 gm = *reinterpret_cast<const uint4 *>(gamma + k0);
            const uint32_t gw[4] = {gm.x, gm.y, gm.z, gm.w};
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t lo = f32_to_bf16_bits(v[j * 8 + 2 * e] * r * __uint_as_float(gw[e] << 16));
                const uint32_t hi = f32_to_bf16_bits(v[j * 8 + 2 * e + 1] * r * __uint_as_float(gw[e] & 0xFFFF0000u));
                w[e] = lo | (hi << 16);
            }
            uint4 o;
            if (pair_order) {
                o.x = prmt(w[0], w[2], 0x5410u);
                o.y = prmt(w[0], w[2], 0x7632u);
                o.z = prmt(w[1], w[3], 0x5410u);
                o.w = prmt(w[1], w[3], 0x7632u);
            } else {
                o = make_uint4(w[0], w[1], w[2], w[3]);
            }
            *reinterpret_cast<uint4 *>(dst + static_cast<int64_t>(m) * ld_dst + k0) = o;
        }
    }
}

}  // namespace qmv

cudaError_t launch_resid_norm(float *h, int64_t ld_h, const float *add, int64_t ld_add, const uint16_t *gamma,
                              float eps, int M, int K, int bits, uint16_t *dst, int64_t ld_dst, cudaStream_t stream,
                              bool pdl) {
    const int per = (K + 2047) / 2048;  // 8 columns per thread per pass, 256 threads
    const int po = bits == 4 ? 1 : 0;
    cudaError_t e;
    switch (per) {
    case 1: e = launch_ex(qmv::resid_norm_kernel<1>, dim3(M), dim3(256), 0, stream, false, pdl, h, ld_h, add, ld_add,
                          gamma, eps, K, po, dst, ld_dst); break;
    case 2: e = launch_ex(qmv::resid_norm_kernel<2>, dim3(M), dim3(256), 0, stream, false, pdl, h, ld_h, add, ld_add,
                          gamma, eps, K, po, dst, ld_dst); break;
    case 3:
    case 4: e = launch_ex(qmv::resid_norm_kernel<4>, dim3(M), dim3(256), 0, stream, false, pdl, h, ld_h, add, ld_add,
                          gamma, eps, K, po, dst, ld_dst); break;
    default: return cudaErrorInvalidValue;
    }
    count_launch();
    return e;
}

bool qmv_supported(const QmmArgs &a, const char **why) {
    auto no = [&](const char *r) { if (why) *why = r; return false; };
    if (a.bits != 4 && a.bits != 8) return no("qmv: bits must be 4 or 8");
    if (a.group != 64) return no("qmv: group_size must be 64");
    if (!a.x_bf16 || !a.p_bf16) return no("qmv: activations and parameters must be bf16");
    if (a.M > kMaxQmvRows) return no("qmv: M > 32");
    if (a.K % (a.bits == 4 ? 256 : 128)) return no("qmv: K must be a multiple of the 128-byte packed stage");
    if (a.x.col_stride != 1 || a.w.col_stride != 1 || a.s.col_stride != 1 || a.b.col_stride != 1)
        return no("qmv: inputs need unit column stride");
    auto al = [](const void *p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    if (!al(a.x.ptr, 16) || a.x.row_stride % 8) return no("qmv: x rows must be 16-byte aligned");
    if (!al(a.w.ptr, 16) || (a.w.row_stride * 4) % 16) return no("qmv: packed rows must be 16-byte aligned");
    if (!al(a.s.ptr, 16) || !al(a.b.ptr, 16) || (a.s.row_stride * 2) % 16 || (a.b.row_stride * 2) % 16)
        return no("qmv: parameter rows must be 16-byte aligned");
    if ((a.N + 159) / 160 > kMaxTiles / 2) return no("qmv: N beyond the arrival-counter region");
    if (a.N >= (int64_t(1) << 31) || a.K >= (int64_t(1) << 30)) return no("qmv: size beyond 32-bit indexing");
    return true;
}

namespace {

constexpr int kSmemCap = 227 * 1024;
constexpr int kOverhead = 1024 + qmv::MAX_STAGES * 4 * qmv::MAX_XR * 4 + 3 * qmv::MAX_STAGES * 8 + 64;

int stage_bytes(int bits, int variant) {
    switch (variant) {
    case 0: return bits == 4 ? qmv::Shape<4, 1, 2, 12>::BYTES : qmv::Shape<8, 1, 2, 12>::BYTES;
    case 1: return bits == 4 ? qmv::Shape<4, 1, 1, 12>::BYTES : qmv::Shape<8, 1, 1, 12>::BYTES;
    case 2: return bits == 4 ? qmv::Shape<4, 2, 2, 10>::BYTES : qmv::Shape<8, 2, 2, 10>::BYTES;
    case 3: return bits == 4 ? qmv::Shape<4, 2, 1, 10>::BYTES : qmv::Shape<8, 2, 1, 10>::BYTES;
    case 5: return bits == 4 ? qmv::Shape<4, 2, 1, 13>::BYTES : qmv::Shape<8, 2, 1, 13>::BYTES;
    default: return bits == 4 ? qmv::Shape<4, 4, 1, 10>::BYTES : qmv::Shape<8, 4, 1, 10>::BYTES;
    }
}

}  // namespace

// Warp-split whole-K plan (qmv_ws_kernel): M <= 16, at most three 16-row
// tiles per SM and at most 32 stages of K; one block of T tiles per CTA, no
// combine across CTAs.  Each CTA streams the whole activation matrix beside
// its 16-48 weight rows, so beyond 32 stages (K 8192 at 4 bits) the stream-K
// plan, whose blocks amortise the activations over 160-320 rows, is faster
// (measured on the 8B down projection, K = 14336: 27 vs 33 us).
static QmvPlan ws_plan(const QmmArgs &a, int num_sms, size_t workspace_bytes) {
    QmvPlan p{};
    if (a.M > 16 || a.K / (a.bits == 4 ? 256 : 128) > 32) return p;
    const int64_t tiles = (a.N + 15) / 16;
    const int T = static_cast<int>((tiles + num_sms - 1) / num_sms);
    if (T > 3) return p;
    const bool mt2 = a.M > 8, b4 = a.bits == 4;
    int bytes, red, kw;
    switch (T) {
    case 1: bytes = qmv::WsShape<4, 2, 1>::BYTES; kw = qmv::WsShape<4, 2, 1>::KW; red = qmv::WsShape<4, 2, 1>::RED; break;
    case 2: bytes = qmv::WsShape<4, 2, 2>::BYTES; kw = qmv::WsShape<4, 2, 2>::KW; red = qmv::WsShape<4, 2, 2>::RED; break;
    default: bytes = qmv::WsShape<4, 2, 3>::BYTES; kw = qmv::WsShape<4, 2, 3>::KW; red = qmv::WsShape<4, 2, 3>::RED; break;
    }
    (void)b4;  // the stage layout does not depend on the code width (128 packed bytes per row)
    if (!mt2) red /= 2;
    const int rows = 16 * T;
    if (qmv::ws_slab_pitch(static_cast<int>(a.K)) > 256) return p;  // one TMA box per slab
    // alignment slack, scale/bias slabs, K-lane sums, group-sum ring
    // (4 groups x 16 rows per slot at most), residual operands (2 KiB per
    // tile), full/empty barriers, the slab and operand barriers, the abort word
    const int overhead = 1024 + qmv::ws_slab_bytes(rows, static_cast<int>(a.K)) + red +
                         qmv::MAX_WS_STAGES * 4 * 16 * 4 + T * 2048 + (2 * qmv::MAX_WS_STAGES + 2) * 8 + 64;
    int stages = std::min(qmv::MAX_WS_STAGES, (kSmemCap - overhead) / bytes);
    stages -= stages % kw;   // every ring slot serves one K lane
    if (stages < 2 * kw) return p;  // group-sum slots are reused only after a later stage's barrier
    const int64_t nblocks = (a.N + rows - 1) / rows;
    const size_t need = kPartialOffset + static_cast<size_t>(nblocks) * a.M * rows * 4 + qmv_prep_bytes(a);
    if (need > workspace_bytes) return p;
    p.splits = 1;
    p.ks = static_cast<int>(a.K);
    p.grid_n = static_cast<int>(nblocks);
    p.stages = stages;
    p.max_slots = 1;
    p.smem_bytes = overhead + stages * bytes;
    p.variant = 5 + T;
    p.rows = rows;
    return p;
}

QmvPlan qmv_plan(const QmmArgs &a, int num_sms, size_t workspace_bytes, bool allow_ws) {
    if (allow_ws) {
        const QmvPlan w = ws_plan(a, num_sms, workspace_bytes);
        if (w.splits) return w;
    }
    // Candidates for this M; each is scored by its makespan in weight
    // row-stages (items per CTA x block rows), with one-tile-per-warp variants
    // charged 12% for their lower activation-fragment reuse (measured consumer
    // rates 64% vs 72% of the HBM rate at M = 16).
    int cand[3], nc = 0;
    if (a.M > 16) {
        cand[nc++] = 4;
    } else if (a.M > 8) {
        cand[nc++] = 2;
        cand[nc++] = 3;
        cand[nc++] = 5;
    } else {
        cand[nc++] = 0;
        cand[nc++] = 1;
    }
    const int kps = a.bits == 4 ? 256 : 128;
    const int64_t spb = a.K / kps;
    QmvPlan best{};
    double best_cost = 0.0;
    for (int ci = 0; ci < nc; ++ci) {
        const int v = cand[ci];
        const int sb = stage_bytes(a.bits, v);
        const int stages = std::min(qmv::MAX_STAGES, (kSmemCap - kOverhead) / sb);
        if (stages < 2) continue;
        const int rows = qmv::kVariantRows[v];
        const int64_t nblocks = (a.N + rows - 1) / rows;
        const int64_t items = nblocks * spb;
        // Variant 5 only as a data-parallel plan: every block whole in one CTA
        // and nearly every SM busy, so no block is combined across CTAs.
        if (v == 5 && (nblocks > num_sms || nblocks * 8 < num_sms * 7)) continue;
        // The fewest CTAs with the makespan of one per SM: fewer contributors
        // per block, less partial traffic (variant 5: one block per CTA).
        const int64_t per_sm = v == 5 ? spb : (items + num_sms - 1) / num_sms;
        const int grid = static_cast<int>((items + per_sm - 1) / per_sm);
        // Contributors per block: a block spans at most ceil(spb / floor(items/grid)) + 1 CTAs.
        const int64_t per_cta = std::max<int64_t>(1, items / grid);
        const int max_slots = static_cast<int>(std::min<int64_t>((spb + per_cta - 1) / per_cta + 1, grid));
        const size_t need = kPartialOffset + static_cast<size_t>(nblocks) * max_slots * a.M * rows * 4 +
                            qmv_prep_bytes(a);
        if (need > workspace_bytes) continue;
        // Plans that combine blocks across CTAs pay for the split-K tail
        // (partial sums written, waited for and re-read: ~20% of a gate/up
        // launch measured).
        const bool shared = items % grid != 0 || (items / grid) % spb != 0;
        const double cost = double(per_sm) * rows * (qmv::kVariantNT[v] == 1 ? 1.12 : 1.0) * (shared ? 1.2 : 1.0);
        if (best.splits && cost >= best_cost) continue;
        QmvPlan p{};
        p.splits = 1;
        p.ks = static_cast<int>(a.K);
        p.grid_n = grid;
        p.stages = stages;
        p.max_slots = max_slots;
        p.smem_bytes = kOverhead + stages * sb;
        p.variant = v;
        p.rows = rows;
        best = p;
        best_cost = cost;
    }
    return best;
}

size_t qmv_prep_bytes(const QmmArgs &a) {
    // 4-bit codes read x in pair order: a converted copy lives at the end of
    // the workspace (aligned to 1 KiB).
    return a.bits == 4 ? ((static_cast<size_t>(a.M) * a.K * 2 + 1023) / 1024) * 1024 : 0;
}

size_t qmv_workspace_bytes(const QmmArgs &a, const QmvPlan &p) {
    const int rows = p.rows;
    const int64_t nblocks = (a.N + rows - 1) / rows;
    return kPartialOffset + static_cast<size_t>(nblocks) * p.max_slots * a.M * rows * 4 + qmv_prep_bytes(a);
}

namespace {
std::atomic<uint64_t> g_arrival_wait_ns{kArrivalWaitNs};
std::atomic<unsigned> g_extra_arrivals{0};
}  // namespace

void qmv_set_combine_wait(uint64_t limit_ns, unsigned extra_arrivals) {
    g_arrival_wait_ns.store(limit_ns ? limit_ns : kArrivalWaitNs);
    g_extra_arrivals.store(extra_arrivals);
}

template <int BITS, int MT, int NT, int CW>
static cudaError_t launch_cfg(const CUtensorMap &wm, const CUtensorMap &sm, const CUtensorMap &bm,
                              const CUtensorMap &xm, const qmv::Params &p, const QmvPlan &plan, cudaStream_t stream,
                              bool pdl) {
    auto kern = qmv::qmv_kernel<BITS, MT, NT, CW>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(kern), plan.smem_bytes);
    if (e != cudaSuccess) return e;
    // Every CTA must be resident for the combine phase: a cooperative launch
    // guarantees it.  With programmatic dependent launch the grid (at most one
    // CTA per SM) becomes resident as the preceding kernel's CTAs leave; the
    // next kernel launches only after every CTA of this grid has started.
    e = launch_ex(kern, dim3(plan.grid_n), dim3(qmv::Shape<BITS, MT, NT, CW>::THREADS), plan.smem_bytes, stream, !pdl,
                  pdl, wm, sm, bm, xm, p);
    count_launch();
    return e;
}

template <int BITS, int MT, int T>
static cudaError_t launch_ws(const CUtensorMap &wm, const CUtensorMap &sm, const CUtensorMap &bm,
                             const CUtensorMap &xm, const qmv::Params &p, const QmvPlan &plan, cudaStream_t stream,
                             bool pdl) {
    auto kern = qmv::qmv_ws_kernel<BITS, MT, T>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(kern), plan.smem_bytes);
    if (e != cudaSuccess) return e;
    // At most one CTA per SM and a grid no larger than the SM count: every
    // CTA is resident (the fused exchange waits on peers' CTAs only).
    e = launch_ex(kern, dim3(plan.grid_n), dim3(qmv::WsShape<BITS, MT, T>::THREADS), plan.smem_bytes, stream, !pdl,
                  pdl, wm, sm, bm, xm, p);
    count_launch();
    return e;
}

cudaError_t launch_qmv_prep(const void *src, int64_t ld_src, int mode, const float *ss, int ss_tiles,
                            const uint16_t *gamma, float eps, int M, int K, int bits, uint16_t *dst, int64_t ld_dst,
                            cudaStream_t stream, bool pdl) {
    const int64_t words = static_cast<int64_t>(M) * (K / 8);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<int64_t>((words + threads - 1) / threads, 1184));
    cudaError_t e = launch_ex(qmv::prep_kernel, dim3(blocks), dim3(threads), 0, stream, false, pdl, src, ld_src, mode,
                              ss, ss_tiles, gamma, eps, M, K, bits == 4 ? 1 : 0, dst, ld_dst);
    count_launch();
    return e;
}

cudaError_t launch_qmv(const QmmArgs &a, const QmvPlan &plan, void *workspace, cudaStream_t stream,
                       const QmvFusion *fusion, bool pdl) {
    if (plan.splits < 1) return cudaErrorInvalidValue;
    qmv::Params p{};
    p.y = a.y;
    p.ldy = a.ldy;
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(a.N);
    p.K = static_cast<int>(a.K);
    const int rows = plan.rows;
    p.nblocks = static_cast<int>((a.N + rows - 1) / rows);
    p.spb = static_cast<int>(a.K / (a.bits == 4 ? 256 : 128));
    p.items = static_cast<int64_t>(p.nblocks) * p.spb;
    p.stages = plan.stages;
    p.max_slots = plan.max_slots;
    p.y_bf16 = a.y_bf16;
    p.arrival_wait_ns = g_arrival_wait_ns.load();
    p.extra_arrivals = g_extra_arrivals.load();
    if (fusion) p.f = *fusion;
    char *ws = static_cast<char *>(workspace);
    p.status = reinterpret_cast<unsigned *>(ws);
    p.counters = reinterpret_cast<unsigned *>(ws + kCounterOffset);
    p.partial = reinterpret_cast<float *>(ws + kPartialOffset);
    // Activations: already in the kernel's order (x_mode 1), or converted
    // into the workspace tail here (4-bit codes need pair order).
    const void *xq = a.x.ptr;
    int64_t ldxq = a.x.row_stride;
    const bool in_order = fusion && fusion->x_mode == 1;
    if (a.bits == 4 && !in_order) {
        uint16_t *dst = reinterpret_cast<uint16_t *>(ws + qmv_workspace_bytes(a, plan) - qmv_prep_bytes(a));
        cudaError_t e = launch_qmv_prep(a.x.ptr, a.x.row_stride, 0, nullptr, 0, nullptr, 0.f, p.M, p.K, 4, dst, p.K,
                                        stream, pdl);
        if (e != cudaSuccess) return e;
        xq = dst;
        ldxq = p.K;
    }
    const CUtensorMap *wm, *sm, *bm, *xm;
    const uint64_t words = static_cast<uint64_t>(a.K) * a.bits / 32;
    if (plan.variant >= 6) {  // warp-split: per-stage packed rows, 3D activation box, per-launch slabs
        const uint32_t rows = static_cast<uint32_t>(plan.rows), sp = qmv::ws_slab_pitch(static_cast<int>(a.K));
        const uint32_t gps = a.bits == 4 ? 4 : 2;
        if (!(wm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w.ptr, words, a.N, a.w.row_stride * 4, 32,
                                        rows, CU_TENSOR_MAP_SWIZZLE_128B)) ||
            !(sm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.s.ptr, a.K / 64, a.N, a.s.row_stride * 2,
                                        sp, rows, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
            !(bm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b.ptr, a.K / 64, a.N, a.b.row_stride * 2,
                                        sp, rows, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
            !(xm = cached_tensor_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xq, 64, a.M, a.K / 64, ldxq * 2, 128, 64, 16,
                                        gps, CU_TENSOR_MAP_SWIZZLE_128B)))
            return cudaErrorInvalidValue;
        const bool b4 = a.bits == 4, mt2 = a.M > 8;
        switch (plan.variant) {
        case 6: return b4 ? (mt2 ? launch_ws<4, 2, 1>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                                 : launch_ws<4, 1, 1>(*wm, *sm, *bm, *xm, p, plan, stream, pdl))
                          : (mt2 ? launch_ws<8, 2, 1>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                                 : launch_ws<8, 1, 1>(*wm, *sm, *bm, *xm, p, plan, stream, pdl));
        case 7: return b4 ? (mt2 ? launch_ws<4, 2, 2>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                                 : launch_ws<4, 1, 2>(*wm, *sm, *bm, *xm, p, plan, stream, pdl))
                          : (mt2 ? launch_ws<8, 2, 2>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                                 : launch_ws<8, 1, 2>(*wm, *sm, *bm, *xm, p, plan, stream, pdl));
        default: return b4 ? (mt2 ? launch_ws<4, 2, 3>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                                  : launch_ws<4, 1, 3>(*wm, *sm, *bm, *xm, p, plan, stream, pdl))
                           : (mt2 ? launch_ws<8, 2, 3>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                                  : launch_ws<8, 1, 3>(*wm, *sm, *bm, *xm, p, plan, stream, pdl));
        }
    }
    const uint32_t xr = a.M > 16 ? 32 : 16;
    const uint32_t box_rows = qmv::kVariantBoxRows[plan.variant];  // 16 rows per consumer warp
    if (!(wm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w.ptr, words, a.N, a.w.row_stride * 4, 32,
                                    box_rows, CU_TENSOR_MAP_SWIZZLE_128B)) ||
        !(sm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.s.ptr, a.K / 64, a.N, a.s.row_stride * 2, 8,
                                    box_rows, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
        !(bm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b.ptr, a.K / 64, a.N, a.b.row_stride * 2, 8,
                                    box_rows, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
        !(xm = cached_tensor_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xq, 64, a.M, a.K / 64, ldxq * 2, 128, 64, xr,
                                    a.bits == 4 ? 4 : 2, CU_TENSOR_MAP_SWIZZLE_128B)))
        return cudaErrorInvalidValue;
    const bool b4 = a.bits == 4;
    switch (plan.variant) {
    case 0: return b4 ? launch_cfg<4, 1, 2, 12>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                      : launch_cfg<8, 1, 2, 12>(*wm, *sm, *bm, *xm, p, plan, stream, pdl);
    case 1: return b4 ? launch_cfg<4, 1, 1, 12>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                      : launch_cfg<8, 1, 1, 12>(*wm, *sm, *bm, *xm, p, plan, stream, pdl);
    case 2: return b4 ? launch_cfg<4, 2, 2, 10>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                      : launch_cfg<8, 2, 2, 10>(*wm, *sm, *bm, *xm, p, plan, stream, pdl);
    case 5: return b4 ? launch_cfg<4, 2, 1, 13>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                      : launch_cfg<8, 2, 1, 13>(*wm, *sm, *bm, *xm, p, plan, stream, pdl);
    case 3: return b4 ? launch_cfg<4, 2, 1, 10>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                      : launch_cfg<8, 2, 1, 10>(*wm, *sm, *bm, *xm, p, plan, stream, pdl);
    default: return b4 ? launch_cfg<4, 4, 1, 10>(*wm, *sm, *bm, *xm, p, plan, stream, pdl)
                       : launch_cfg<8, 4, 1, 10>(*wm, *sm, *bm, *xm, p, plan, stream, pdl);
    }
}

}  // namespace afb
