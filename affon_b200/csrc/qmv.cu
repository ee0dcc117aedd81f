// Decode qmv for sm_100a: y[M,N] = x[M,K] . decode(W)[N,K]^T for M <= 16,
// 4- or 8-bit codes packed little-endian into u32 along K, group 64, bf16
// activations / scales / biases, f32 accumulation (the layout and formula of
// docs/core/quantized-inference.md:45-67).
//
// Streaming.  Persistent CTAs, one per SM.  One producer warp moves the
// packed weight matrix through a ring of shared-memory stages with 2D TMA
// loads (ROWS rows x 128 bytes per stage, 128-byte swizzle, plus the matching
// ROWS x 8 boxes of bf16 scales and biases), so ~120 KB per SM are in flight
// without costing registers.  Consumer warps read the packed words from
// shared memory, decode them in registers and feed tensor cores.
//
// Why tensor cores at M <= 16: at ~6.5 TB/s a 4-bit weight stream delivers
// ~11.6e12 weights/s; decoding each weight to a float and multiplying it on
// the CUDA cores costs ~3 lane-ops, as much as the 148 SMs can issue.  The
// decoded codes go straight from registers into the A fragments of
// m16n8k16 bf16 MMAs (weights as the 16-row A operand, activations as B).
// Shifts of the nibble decoder are issued as mul.hi so they run on the FMA
// pipe beside the logic ops on the ALU pipe.
//
// Exact codes, per-group affine in f32: the MMA multiplies the integer codes
// (4-bit: as 128+q, exact in bf16) by x, giving C_g = sum_{k in g} x*code in
// f32; the affine decode is applied per group of 64 outside the tensor core:
//     y += s[n,g] * C_g + (b[n,g] - 128 s[n,g]) * X_g,  X_g = sum_{k in g} x[k]
// evaluated as fused multiply-adds so the offset terms cancel exactly.  This
// is sum_k x*(s*q+b) up to reassociation; weights are never rounded to bf16
// (quantized-inference.md:119-121).  Numerical class: reassociated.
//
// Work partition (stream-K).  The work is a flat list of items
// (K split, 16*NT*CW-row block, 128-byte K stage), split-major.  CTA c takes
// the items [c*T/C, (c+1)*T/C), so every CTA streams the same number of
// bytes.  K is split where x would not fit in shared memory and, beyond that,
// where staging x in every CTA would cost more on-chip traffic than the extra
// partial sums; a CTA restages x when its range enters a new split.  A block
// that lies inside one CTA and one split is stored directly; a block shared
// by several CTAs or splits is combined through f32 partials: each
// contributing CTA writes its slot, and the CTA arriving last (per-block
// counter) sums the slots in a fixed order and stores y, so results do not
// depend on scheduling.  That CTA resets the counter for the next launch.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace afb {
namespace qmv {

constexpr int GROUP = 64;
constexpr int XS_PAD = 8;
constexpr int MAX_STAGES = 8;

template <int NT, int CW>
struct Geom {
    static constexpr int ROWS = 16 * NT * CW;   // rows per block (= TMA box height)
    static constexpr int W_BYTES = ROWS * 128;  // packed bytes per stage
    static constexpr int SB_BYTES = ROWS * 16;  // one 8-group box of scales (or biases)
    static constexpr int STAGE_BYTES = W_BYTES + 2 * SB_BYTES;
};

template <int BITS>
struct Shape {
    static constexpr int GPS = BITS == 4 ? 4 : 2;  // groups per stage (128 packed bytes per row)
    static constexpr int KPS = GPS * GROUP;         // K per stage
};

struct Params {
    const uint16_t *x;
    int64_t ldx;
    void *y;
    int64_t ldy;
    float *partial;
    unsigned *counters;
    unsigned *status;
    int M, N, K;
    int splits, ks;       // K splits (x slices that fit shared memory) and K per split
    int nblocks, spb;     // blocks along N and stages per block per split
    int64_t items;        // splits * nblocks * spb
    int stages;           // ring depth
    int max_slots;        // partial slots per block
    int y_bf16;
    QmvFusion f;
};

__device__ __forceinline__ uint32_t shr_fma_pipe(uint32_t w, int s) {
    uint32_t r;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(r) : "r"(w), "r"(1u << (32 - s)));
    return r;
}
// Codes p and p+4 of a 4-bit word as the exact bf16 pair (128+q_p, 128+q_{p+4}).
__device__ __forceinline__ uint32_t dec4(uint32_t w, int p) {
    return lop3_and_or(p ? shr_fma_pipe(w, 4 * p) : w, 0x000F000Fu, 0x43004300u);
}
// Bytes i and i+1 of an 8-bit word as an exact bf16 pair (via 2^23 + q in f32).
__device__ __forceinline__ uint32_t dec8(uint32_t w, int i) {
    float f0 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i)) - 8388608.0f;
    float f1 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i + 1)) - 8388608.0f;
    return pack_bf16x2(f0, f1);
}

__device__ __forceinline__ void store_out(const Params &p, int m, int64_t n, float v) {
    if (p.y_bf16)
        static_cast<uint16_t *>(p.y)[m * p.ldy + n] = f32_to_bf16_bits(v);
    else
        static_cast<float *>(p.y)[m * p.ldy + n] = v;
}

__device__ __forceinline__ const float *base_of_slot(const float *base, int slot, int M, int rows) {
    return base + static_cast<int64_t>(slot) * M * rows;
}

// Owner CTA of flat item i when CTA c holds [floor(c*T/C), floor((c+1)*T/C)).
__device__ __forceinline__ int owner_of(int64_t i, int64_t T, int C) {
    return static_cast<int>(((i + 1) * C - 1) / T);
}

// Contributor count of block blk (all splits) and the slot of CTA c for split.
__device__ __forceinline__ void contributors(const Params &p, int split, int blk, int c, int C, int &total,
                                             int &slot) {
    total = 0;
    slot = -1;
    for (int s = 0; s < p.splits; ++s) {
        const int64_t b0 = (static_cast<int64_t>(s) * p.nblocks + blk) * p.spb;
        const int first = owner_of(b0, p.items, C), last = owner_of(b0 + p.spb - 1, p.items, C);
        if (s == split) slot = total + (c - first);
        total += last - first + 1;
    }
}

__device__ __forceinline__ uint32_t f32_order_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Apply the epilogue to the row pair (n_lo, n_lo + 8) of activation row m.
// Returns the contribution of this pair to the per-tile reductions:
// EPI_RESID: sum of squares of the updated residual entries; EPI_ARGMAX: the
// packed best (key << 32 | ~n) of the pair.  Rows at or beyond N are skipped.
__device__ __forceinline__ unsigned long long epilogue_pair(const Params &p, int m, int64_t n_lo, float v_lo,
                                                            float v_hi, float &ssq) {
    const int64_t n_hi = n_lo + 8;
    const bool ok_lo = n_lo < p.N, ok_hi = n_hi < p.N;
    unsigned long long best = 0ull;
    switch (p.f.epi) {
    case EPI_RESID: {
        float *h = p.f.h_out + m * p.f.ld_h_out;
        if (ok_lo) { const float hv = h[n_lo] + v_lo; h[n_lo] = hv; ssq = fmaf(hv, hv, ssq); }
        if (ok_hi) { const float hv = h[n_hi] + v_hi; h[n_hi] = hv; ssq = fmaf(hv, hv, ssq); }
        break;
    }
    case EPI_SILU_MUL:
        if (ok_hi) {  // tile rows 0-7 are gate rows, 8-15 the matching up rows
            const int64_t j = (n_lo >> 4) * 8 + (n_lo & 7);
            const float gate = v_lo;
            const float silu = gate / (1.0f + __expf(-gate));
            p.f.act[m * p.f.ld_act + j] = f32_to_bf16_bits(silu * v_hi);
        }
        break;
    case EPI_ARGMAX:
        if (ok_lo) best = (static_cast<unsigned long long>(f32_order_key(v_lo)) << 32) | (0xFFFFFFFFu - uint32_t(n_lo));
        if (ok_hi) {
            const unsigned long long c =
                (static_cast<unsigned long long>(f32_order_key(v_hi)) << 32) | (0xFFFFFFFFu - uint32_t(n_hi));
            best = c > best ? c : best;
        }
        break;
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
        if (lead && m < p.M) p.f.ss_out[tile * 16 + m] = ssq;
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
template <int MT>
__device__ __forceinline__ void finish_tile(const Params &p, const float (&v)[MT][4], int64_t n0, int g, int t) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = 2 * t + 8 * mt + h;
            float ssq = 0.0f;
            unsigned long long best = 0ull;
            if (m < p.M) best = epilogue_pair(p, m, n0 + g, v[mt][h], v[mt][2 + h], ssq);
            publish_tile(p, n0 >> 4, m, g == 0, ssq, best);
        }
}

// Epilogue of one (split, block) segment of this CTA for the warp's NT tiles.
// Called by all consumer warps together.  `flag` is a shared-memory word.
template <int MT, int NT, int CW>
__device__ __forceinline__ void segment_epilogue(const Params &p, float (&acc)[NT][MT][4], int split, int blk, int warp,
                                                 int g, int t, int lane, int tid, volatile int *flag) {
    constexpr int ROWS = Geom<NT, CW>::ROWS;
    int total, slot;
    contributors(p, split, blk, blockIdx.x, gridDim.x, total, slot);
    const int64_t nb0 = static_cast<int64_t>(blk) * ROWS;
    if (total == 1) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) finish_tile<MT>(p, acc[nt], nb0 + (warp * NT + nt) * 16, g, t);
        return;
    }
    // partial[((blk * max_slots + slot) * M + m) * ROWS + row]
    float *base = p.partial + (static_cast<int64_t>(blk) * p.max_slots) * p.M * ROWS;
    float *const base_ptr = base;
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
    // Message passing through the per-block counter (one arrival per
    // contributing CTA): every thread releases its partials with a gpu-scope
    // acq_rel fence, the consumer warps meet, one thread takes the ticket,
    // and in the last contributor every thread fences again before reading
    // all slots.
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    named_bar_sync(1, CW * 32);
    if (tid == 0) *flag = (atomicAdd(&p.counters[blk], 1u) == static_cast<unsigned>(total - 1)) ? 1 : 0;
    named_bar_sync(1, CW * 32);
    const bool last = *flag != 0;
    named_bar_sync(1, CW * 32);  // the flag is reused by the next segment
    if (!last) return;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    // Each warp reduces the rows it owns, lanes over (row, row+8) pairs of its
    // tiles so the pair epilogues and per-tile reductions apply unchanged.
    for (int base = warp * 8 * NT; base < (warp + 1) * 8 * NT; base += 32) {
        const int pr = base + lane;
        const bool active = pr < (warp + 1) * 8 * NT;
        const int r_lo = (pr >> 3) * 16 + (pr & 7);
        for (int m = 0; m < p.M; ++m) {
            float ssq = 0.0f;
            unsigned long long best = 0ull;
            if (active) {
                float lo = 0.0f, hi = 0.0f;
                for (int sl = 0; sl < total; ++sl) {
                    const float *slot_base = base_of_slot(base_ptr, sl, p.M, ROWS) + static_cast<int64_t>(m) * ROWS;
                    lo += __ldcg(&slot_base[r_lo]);
                    hi += __ldcg(&slot_base[r_lo + 8]);
                }
                best = epilogue_pair(p, m, nb0 + r_lo, lo, hi, ssq);
            }
            // lanes pr..pr+7 share a tile: reduce over the low 3 lane bits
            if (p.f.epi == EPI_RESID) {
                ssq += __shfl_xor_sync(0xffffffffu, ssq, 1);
                ssq += __shfl_xor_sync(0xffffffffu, ssq, 2);
                ssq += __shfl_xor_sync(0xffffffffu, ssq, 4);
                if (active && (pr & 7) == 0) p.f.ss_out[((nb0 + r_lo) >> 4) * 16 + m] = ssq;
            } else if (p.f.epi == EPI_ARGMAX) {
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                    best = other > best ? other : best;
                }
                if (active && (pr & 7) == 0 && best) atomicMax(&p.f.amax[m], best);
            }
        }
    }
    if (tid == 0) atomicExch(&p.counters[blk], 0u);
}

// Stage x[:, k0:k0+ks) (and the group sums X_g) into shared memory; run by
// the consumer warps only.
template <int BITS>
__device__ __forceinline__ void stage_x(const Params &p, char *xs, float *xg, int xs_rs, int64_t k0, int tid,
                                        int nthreads, float *rms, float *red) {
    const int gs = p.ks / GROUP;
    for (int i = tid; i < gs * 16; i += nthreads) xg[i] = 0.0f;
    if (p.f.x_mode == 1) {
        // 1/rms of every activation row from the per-tile sums of squares
        // (fixed summation order: per thread, then per warp, then per CTA).
        float acc[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) acc[m] = 0.0f;
        for (int tl = tid; tl < p.f.ss_tiles; tl += nthreads) {
            const float4 *src = reinterpret_cast<const float4 *>(p.f.ss_in + static_cast<int64_t>(tl) * 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = __ldcg(src + q);
                acc[4 * q] += v.x; acc[4 * q + 1] += v.y; acc[4 * q + 2] += v.z; acc[4 * q + 3] += v.w;
            }
        }
        const int lane = tid & 31, w = tid >> 5;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
#pragma unroll
            for (int o = 16; o; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
            if (lane == 0) red[w * 16 + m] = acc[m];
        }
        named_bar_sync(1, nthreads);
        if (tid < 16) {
            float sum = 0.0f;
            for (int ww = 0; ww < nthreads / 32; ++ww) sum += red[ww * 16 + tid];
            rms[tid] = rsqrtf(sum / static_cast<float>(p.K) + p.f.eps);
        }
    }
    named_bar_sync(1, nthreads);
    const int cpr = p.ks / 8;  // 16-byte chunks per row
    const int total = p.M * cpr;
    for (int base = 0; base < total; base += nthreads) {
        const int c = base + tid;
        const bool valid = c < total;
        const int m = valid ? c / cpr : 0, kc = valid ? c % cpr : 0;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) {
            if (p.f.x_mode == 1) {  // x = bf16(h * rms * gamma)
                const float4 *hp = reinterpret_cast<const float4 *>(p.f.h_in + m * p.f.ld_h_in + k0 + kc * 8);
                const float4 h0 = __ldcg(hp), h1 = __ldcg(hp + 1);
                const uint4 gm = ldg_nc_v4(p.f.gamma + k0 + kc * 8);
                const float r = rms[m];
                auto nb = [&](float hv, uint32_t gw, int hi) {
                    return f32_to_bf16_bits(hv * r * bf16_bits_to_f32(hi ? (gw >> 16) : (gw & 0xFFFF)));
                };
                v.x = nb(h0.x, gm.x, 0) | (uint32_t(nb(h0.y, gm.x, 1)) << 16);
                v.y = nb(h0.z, gm.y, 0) | (uint32_t(nb(h0.w, gm.y, 1)) << 16);
                v.z = nb(h1.x, gm.z, 0) | (uint32_t(nb(h1.y, gm.z, 1)) << 16);
                v.w = nb(h1.z, gm.w, 0) | (uint32_t(nb(h1.w, gm.w, 1)) << 16);
            } else {
                v = ldg_nc_v4(p.x + m * p.ldx + k0 + kc * 8);
            }
        }
        float sum = bf16_bits_to_f32(v.x & 0xFFFF) + bf16_bits_to_f32(v.x >> 16) + bf16_bits_to_f32(v.y & 0xFFFF) +
                    bf16_bits_to_f32(v.y >> 16) + bf16_bits_to_f32(v.z & 0xFFFF) + bf16_bits_to_f32(v.z >> 16) +
                    bf16_bits_to_f32(v.w & 0xFFFF) + bf16_bits_to_f32(v.w >> 16);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (valid) {
            if constexpr (BITS == 4) {  // [x0 x4 x1 x5 x2 x6 x3 x7] matches dec4's pairs
                uint4 o;
                o.x = prmt(v.x, v.z, 0x5410u);
                o.y = prmt(v.x, v.z, 0x7632u);
                o.z = prmt(v.y, v.w, 0x5410u);
                o.w = prmt(v.y, v.w, 0x7632u);
                v = o;
            }
            *reinterpret_cast<uint4 *>(xs + m * xs_rs + kc * 16) = v;
            if ((kc & 7) == 0) xg[(kc >> 3) * 16 + m] = sum;
        }
    }
    named_bar_sync(1, nthreads);
}

template <int BITS, int MT, int NT, int CW>
__global__ void __launch_bounds__(32 * (CW + 1), 1)
    qmv_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
               const __grid_constant__ CUtensorMap bmap, Params p) {
    using Gm = Geom<NT, CW>;
    constexpr int STAGE_BYTES = Gm::STAGE_BYTES, W_BYTES = Gm::W_BYTES, SB_BYTES = Gm::SB_BYTES, ROWS = Gm::ROWS;
    constexpr int GPS = Shape<BITS>::GPS, KPS = Shape<BITS>::KPS;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    char *ring = smem;
    const int xs_rs = (p.ks + XS_PAD) * 2;
    char *xs = ring + S * STAGE_BYTES;
    float *xg = reinterpret_cast<float *>(xs + p.M * xs_rs);
    uint64_t *full = reinterpret_cast<uint64_t *>(xg + (p.ks / GROUP) * 16);
    uint64_t *empty = full + MAX_STAGES;
    volatile int *abort = reinterpret_cast<volatile int *>(empty + MAX_STAGES);
    volatile int *flag = abort + 1;
    float *rms = reinterpret_cast<float *>(empty + MAX_STAGES) + 4;  // [16]
    float *red = rms + 16;                                            // [CW][16]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const int64_t T = p.items;
    const int64_t lo = static_cast<int64_t>(blockIdx.x) * T / gridDim.x;
    const int64_t hi = static_cast<int64_t>(blockIdx.x + 1) * T / gridDim.x;
    const int64_t per_split = static_cast<int64_t>(p.nblocks) * p.spb;

    if (warp == CW) {  // ------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            tma_prefetch_desc(&smap);
            tma_prefetch_desc(&bmap);
            int stage = 0;
            uint32_t phase = 0;
            for (int64_t i = lo; i < hi; ++i) {
                const int split = static_cast<int>(i / per_split);
                const int64_t rem = i - split * per_split;
                const int blk = static_cast<int>(rem / p.spb), st = static_cast<int>(rem - int64_t(blk) * p.spb);
                // On a timed-out wait (abort set) stop issuing loads; consumers drain.
                if (!mbar_wait(&empty[stage], phase ^ 1, abort, p.status)) return;
                char *dst = ring + stage * STAGE_BYTES;
                mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                const int64_t kk = static_cast<int64_t>(split) * p.ks + static_cast<int64_t>(st) * KPS;
                tma_load_2d(dst, &wmap, &full[stage], static_cast<int>(kk * BITS / 32), blk * ROWS);
                const int g8 = static_cast<int>((kk / GROUP) & ~int64_t(7));
                tma_load_2d(dst + W_BYTES, &smap, &full[stage], g8, blk * ROWS);
                tma_load_2d(dst + W_BYTES + SB_BYTES, &bmap, &full[stage], g8, blk * ROWS);
                if (++stage == S) { stage = 0; phase ^= 1; }
            }
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    const int g = lane >> 2, t = lane & 3;
    int stage = 0;
    uint32_t phase = 0;
    int cur_split = -1;
    int64_t i = lo;
    while (i < hi) {
        const int split = static_cast<int>(i / per_split);
        const int64_t rem = i - split * per_split;
        const int blk = static_cast<int>(rem / p.spb);
        const int64_t blk_begin = static_cast<int64_t>(split) * per_split + static_cast<int64_t>(blk) * p.spb;
        const int64_t seg_end = min(hi, blk_begin + p.spb);
        if (split != cur_split) {
            named_bar_sync(1, CW * 32);
            stage_x<BITS>(p, xs, xg, xs_rs, static_cast<int64_t>(split) * p.ks, tid, CW * 32, rms, red);
            cur_split = split;
        }
        float acc[NT][MT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) acc[nt][mt][0] = acc[nt][mt][1] = acc[nt][mt][2] = acc[nt][mt][3] = 0.f;

        for (; i < seg_end; ++i) {
            const int j = static_cast<int>(i - blk_begin);  // stage index within the block
            // A timed-out wait sets *abort; keep walking the loop (results are
            // then garbage and the status word says TIMEOUT) so that every
            // consumer reaches the same named barriers and no thread hangs.
            mbar_wait(&full[stage], phase, abort, p.status);
            const char *sw = ring + stage * STAGE_BYTES;
            const char *ssb = sw + W_BYTES;
            const char *bsb = ssb + SB_BYTES;
            const int go0 = (j * GPS) & 7;  // first group of this stage within the 8-group scale box
            uint32_t sv[NT][2][GPS / 2], bv[NT][2][GPS / 2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = (warp * NT + nt) * 16 + g + 8 * h;
                    if constexpr (GPS == 4) {
                        const uint2 a = *reinterpret_cast<const uint2 *>(ssb + r * 16 + go0 * 2);
                        const uint2 b = *reinterpret_cast<const uint2 *>(bsb + r * 16 + go0 * 2);
                        sv[nt][h][0] = a.x; sv[nt][h][1] = a.y; bv[nt][h][0] = b.x; bv[nt][h][1] = b.y;
                    } else {
                        sv[nt][h][0] = *reinterpret_cast<const uint32_t *>(ssb + r * 16 + go0 * 2);
                        bv[nt][h][0] = *reinterpret_cast<const uint32_t *>(bsb + r * 16 + go0 * 2);
                    }
                }
#pragma unroll
            for (int G = 0; G < GPS; ++G) {
                const int Gl = j * GPS + G;  // group index within the split
                uint32_t xf[MT][8];
                float2 X[MT];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const int m = g + 8 * mt;
                    if (m < p.M) {
                        const char *src = xs + m * xs_rs + (Gl * GROUP + 16 * t) * 2;
                        const uint4 v0 = *reinterpret_cast<const uint4 *>(src);
                        const uint4 v1 = *reinterpret_cast<const uint4 *>(src + 16);
                        xf[mt][0] = v0.x; xf[mt][1] = v0.y; xf[mt][2] = v0.z; xf[mt][3] = v0.w;
                        xf[mt][4] = v1.x; xf[mt][5] = v1.y; xf[mt][6] = v1.z; xf[mt][7] = v1.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) xf[mt][e] = 0u;
                    }
                    X[mt] = *reinterpret_cast<const float2 *>(xg + Gl * 16 + 2 * t + 8 * mt);
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int r0 = (warp * NT + nt) * 16 + g;  // block row of this thread (and r0 + 8)
                    uint32_t w0[4], w1[4];
                    if constexpr (BITS == 4) {
                        const int off = (((2 * G + (t >> 1)) ^ g) << 4) + (t & 1) * 8;
                        const uint2 a = *reinterpret_cast<const uint2 *>(sw + r0 * 128 + off);
                        const uint2 b = *reinterpret_cast<const uint2 *>(sw + (r0 + 8) * 128 + off);
                        w0[0] = a.x; w0[1] = a.y; w1[0] = b.x; w1[1] = b.y;
                    } else {
                        const int off = ((4 * G + t) ^ g) << 4;
                        const uint4 a = *reinterpret_cast<const uint4 *>(sw + r0 * 128 + off);
                        const uint4 b = *reinterpret_cast<const uint4 *>(sw + (r0 + 8) * 128 + off);
                        w0[0] = a.x; w0[1] = a.y; w0[2] = a.z; w0[3] = a.w;
                        w1[0] = b.x; w1[1] = b.y; w1[2] = b.z; w1[3] = b.w;
                    }
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
                    float c[MT][4];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) c[mt][0] = c[mt][1] = c[mt][2] = c[mt][3] = 0.f;
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        uint32_t a[4], b0[MT], b1[MT];
                        if constexpr (BITS == 4) {
                            const int p0 = 2 * (s & 1);
                            const uint32_t u0 = w0[s >> 1], u1 = w1[s >> 1];
                            a[0] = dec4(u0, p0);
                            a[1] = dec4(u1, p0);
                            a[2] = dec4(u0, p0 + 1);
                            a[3] = dec4(u1, p0 + 1);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                b0[mt] = xf[mt][4 * (s >> 1) + p0];
                                b1[mt] = xf[mt][4 * (s >> 1) + p0 + 1];
                            }
                        } else {
                            a[0] = dec8(w0[s], 0);
                            a[1] = dec8(w1[s], 0);
                            a[2] = dec8(w0[s], 2);
                            a[3] = dec8(w1[s], 2);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                b0[mt] = xf[mt][2 * s];
                                b1[mt] = xf[mt][2 * s + 1];
                            }
                        }
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) mma_bf16_16816(c[mt], a, b0[mt], b1[mt], c[mt]);
                    }
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        acc[nt][mt][0] = fmaf(s0, c[mt][0], fmaf(q0, X[mt].x, acc[nt][mt][0]));
                        acc[nt][mt][1] = fmaf(s0, c[mt][1], fmaf(q0, X[mt].y, acc[nt][mt][1]));
                        acc[nt][mt][2] = fmaf(s1, c[mt][2], fmaf(q1, X[mt].x, acc[nt][mt][2]));
                        acc[nt][mt][3] = fmaf(s1, c[mt][3], fmaf(q1, X[mt].y, acc[nt][mt][3]));
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
        segment_epilogue<MT, NT, CW>(p, acc, split, blk, warp, g, t, lane, tid, flag);
    }
}

}  // namespace qmv

bool qmv_supported(const QmmArgs &a, const char **why) {
    auto no = [&](const char *r) { if (why) *why = r; return false; };
    if (a.bits != 4 && a.bits != 8) return no("qmv: bits must be 4 or 8");
    if (a.group != 64) return no("qmv: group_size must be 64");
    if (!a.x_bf16 || !a.p_bf16) return no("qmv: activations and parameters must be bf16");
    if (a.M > 16) return no("qmv: M > 16");
    if (a.K % 512) return no("qmv: K must be a multiple of 512");
    if (a.x.col_stride != 1 || a.w.col_stride != 1 || a.s.col_stride != 1 || a.b.col_stride != 1)
        return no("qmv: inputs need unit column stride");
    auto al = [](const void *p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    if (!al(a.x.ptr, 16) || a.x.row_stride % 8) return no("qmv: x rows must be 16-byte aligned");
    if (!al(a.w.ptr, 16) || (a.w.row_stride * 4) % 16) return no("qmv: packed rows must be 16-byte aligned");
    if (!al(a.s.ptr, 16) || !al(a.b.ptr, 16) || (a.s.row_stride * 2) % 16 || (a.b.row_stride * 2) % 16)
        return no("qmv: parameter rows must be 16-byte aligned");
    if ((a.N + 255) / 256 > kMaxTiles) return no("qmv: N beyond the arrival-counter region");
    if (a.N >= (int64_t(1) << 31) || a.K >= (int64_t(1) << 30)) return no("qmv: size beyond 32-bit indexing");
    return true;
}

namespace {

// M <= 8: one column tile, 16 consumer warps of one 16-row tile each
// (256-row blocks).  M > 8: two column tiles; 8 consumer warps of two 16-row
// tiles each (256-row blocks) so each activation fragment feeds two tiles.
struct Variant {
    int nt, cw, rows, stage_bytes;
};
Variant variant_of(const QmmArgs &a) {
    if (a.M > 8) return {2, 8, qmv::Geom<2, 8>::ROWS, qmv::Geom<2, 8>::STAGE_BYTES};
    return {1, 16, qmv::Geom<1, 16>::ROWS, qmv::Geom<1, 16>::STAGE_BYTES};
}

int x_bytes(const QmmArgs &a, int ks) { return static_cast<int>(a.M) * (ks + qmv::XS_PAD) * 2 + (ks / 64) * 16 * 4; }

constexpr int kSmemCap = 227 * 1024;
constexpr int kMinRing = 2 * 40 * 1024;   // keep >= 80 KB of weights in flight
constexpr int kMaxRing = 128 * 1024;

}  // namespace

QmvPlan qmv_plan(const QmmArgs &a, int num_sms, size_t workspace_bytes) {
    QmvPlan p{};
    const Variant v = variant_of(a);
    const int nk = static_cast<int>(a.K / 512);
    const int overhead = 1024 + 2 * qmv::MAX_STAGES * 8 + 64 + 20 * 16 * 4;
    // K splits: the smallest count whose x slice fits next to the ring, raised
    // towards the count that balances the two on-chip costs of stream-K --
    // every CTA stages its x slice (grid * M * K/S * 2 bytes) while every
    // extra split adds partial sums (about 8 * S * M * N bytes) -- which is
    // minimised near S = sqrt(grid * K / (4 * N)).
    int smin = 0;
    for (int s = 1; s <= nk; ++s) {
        if (nk % s) continue;
        if (overhead + x_bytes(a, static_cast<int>(a.K / s)) + std::max(kMinRing, 2 * v.stage_bytes) <= kSmemCap) {
            smin = s;
            break;
        }
    }
    if (smin == 0) return p;
    const double s_opt = std::sqrt(static_cast<double>(num_sms) * a.K / (4.0 * a.N));
    int splits = smin;
    for (int s = smin; s <= nk; ++s)
        if (nk % s == 0 && s <= s_opt * 1.5) splits = s;
    const int ks = static_cast<int>(a.K / splits);
    const int ring_room = kSmemCap - overhead - x_bytes(a, ks);
    const int stages = std::min(qmv::MAX_STAGES, std::min(ring_room, kMaxRing) / v.stage_bytes);
    if (stages < 2) return p;
    const int64_t nblocks = (a.N + v.rows - 1) / v.rows;
    const int kps = a.bits == 4 ? 256 : 128;
    const int64_t spb = ks / kps;
    const int64_t items = nblocks * spb * splits;
    const int grid = static_cast<int>(std::min<int64_t>(num_sms, items));
    // Upper bound of contributors per block: per split, a block spans at most
    // ceil(spb / floor(items/grid)) + 1 CTAs.
    const int64_t per_cta = std::max<int64_t>(1, items / grid);
    const int max_slots = static_cast<int>(splits * ((spb + per_cta - 1) / per_cta + 1));
    const size_t need = kPartialOffset + static_cast<size_t>(nblocks) * max_slots * a.M * v.rows * 4;
    if (need > workspace_bytes) return p;
    p.splits = splits;
    p.ks = ks;
    p.grid_n = grid;
    p.stages = stages;
    p.max_slots = max_slots;
    p.smem_bytes = overhead + x_bytes(a, ks) + stages * v.stage_bytes;
    return p;
}

size_t qmv_workspace_bytes(const QmmArgs &a, const QmvPlan &p) {
    const Variant v = variant_of(a);
    const int64_t nblocks = (a.N + v.rows - 1) / v.rows;
    return kPartialOffset + static_cast<size_t>(nblocks) * p.max_slots * a.M * v.rows * 4;
}

template <int BITS, int MT, int NT, int CW>
static cudaError_t launch_cfg(const CUtensorMap &wm, const CUtensorMap &sm, const CUtensorMap &bm,
                              const qmv::Params &p, const QmvPlan &plan, cudaStream_t stream) {
    auto kern = qmv::qmv_kernel<BITS, MT, NT, CW>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(kern), plan.smem_bytes);
    if (e != cudaSuccess) return e;
    kern<<<plan.grid_n, 32 * (CW + 1), plan.smem_bytes, stream>>>(wm, sm, bm, p);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_qmv(const QmmArgs &a, const QmvPlan &plan, void *workspace, cudaStream_t stream,
                       const QmvFusion *fusion) {
    if (plan.splits < 1) return cudaErrorInvalidValue;
    const Variant v = variant_of(a);
    qmv::Params p{};
    p.x = static_cast<const uint16_t *>(a.x.ptr);
    p.ldx = a.x.row_stride;
    p.y = a.y;
    p.ldy = a.ldy;
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(a.N);
    p.K = static_cast<int>(a.K);
    p.splits = plan.splits;
    p.ks = plan.ks;
    p.nblocks = static_cast<int>((a.N + v.rows - 1) / v.rows);
    p.spb = plan.ks / (a.bits == 4 ? 256 : 128);
    p.items = static_cast<int64_t>(p.nblocks) * p.spb * p.splits;
    p.stages = plan.stages;
    p.max_slots = plan.max_slots;
    p.y_bf16 = a.y_bf16;
    if (fusion) p.f = *fusion;
    char *ws = static_cast<char *>(workspace);
    p.status = reinterpret_cast<unsigned *>(ws);
    p.counters = reinterpret_cast<unsigned *>(ws + kCounterOffset);
    p.partial = reinterpret_cast<float *>(ws + kPartialOffset);
    const CUtensorMap *wm, *sm, *bm;
    const uint64_t words = static_cast<uint64_t>(a.K) * a.bits / 32;
    if (!(wm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w.ptr, words, a.N, a.w.row_stride * 4, 32, v.rows,
                                    CU_TENSOR_MAP_SWIZZLE_128B)) ||
        !(sm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.s.ptr, a.K / 64, a.N, a.s.row_stride * 2, 8,
                                    v.rows, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
        !(bm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b.ptr, a.K / 64, a.N, a.b.row_stride * 2, 8,
                                    v.rows, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return cudaErrorInvalidValue;
    if (a.M > 8)
        return a.bits == 4 ? launch_cfg<4, 2, 2, 8>(*wm, *sm, *bm, p, plan, stream)
                           : launch_cfg<8, 2, 2, 8>(*wm, *sm, *bm, p, plan, stream);
    return a.bits == 4 ? launch_cfg<4, 1, 1, 16>(*wm, *sm, *bm, p, plan, stream)
                       : launch_cfg<8, 1, 1, 16>(*wm, *sm, *bm, p, plan, stream);
}

}  // namespace afb
