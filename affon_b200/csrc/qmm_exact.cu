// Prefill qmm for sm_100a with reassociated numerics (the reference's default
// `backend_equivalent` contract): y[M,N] = x[M,K] . decode(W)[N,K]^T for
// large M, 4/8-bit codes packed little-endian into u32 along K, group 64,
// bf16 x / scales / biases, f32 (or bf16) result.  Weights are never rounded:
//
//     y[m,n] = sum_g s[n,g] * C_g[n,m]  +  sum_g b[n,g] * X[m,g]
//     C_g[n,m] = sum_{k in g} q[n,k] * x[m,k]     (exact integer codes q)
//     X[m,g]   = sum_{k in g} x[m,k]
//
// which is sum_k x*(s*q + b) up to reassociation
// (docs/core/quantized-inference.md:57,114-128: f32 accumulation, class
// `reassociated`).
//
// Tensor cores.  The exact codes (0..15 or 0..255, exact in bf16) are the
// A operand (128 weight rows, K-major, 128-byte swizzle) and the activation
// tile the B operand (256 activation rows), so each decoded code feeds 256
// rows.  Every 64-wide K group accumulates alone into one of two TMEM
// accumulators (128 lanes x 256 f32 columns each, all 512 columns), so the
// tensor core computes group g+1 while the f32 scale of group g is applied
// on the CUDA cores.
//
// The bias term on tensor cores.  sum_g b[n,g] X[m,g] is itself a small
// matrix product over the group index.  A prep kernel writes X[m,g] as three
// bf16 pieces hi + mid + lo whose sum is X exactly (24 significant bits),
// three columns per group, 21 groups per 64-column stage, in an [M, KB3]
// activation side array (KB3 = 64 ceil(G / 21), zero padded); the weight
// side repeats b[n,g] (exact in bf16) at the same three columns.  Products of
// bf16 values are exact in f32, so one extra accumulation unit of KB3/64
// stages per tile (about 1/21 more MMA work) forms the bias term in f32, and
// the epilogue adds it with scale 1.
//
// Warp roles (512 threads, one persistent CTA per SM):
//   warp 0      TMA producer: activation tiles, then the X pieces per tile
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warp 2      TMA producer of packed-weight tiles
//   warp 3      idle
//   warps 4-7   dequantisers, one weight row each: packed words -> exact
//               bf16 codes in the swizzled A tile; for the bias stages,
//               b[n,g] repeated three times
//   warps 8-15  epilogue, one weight row n (TMEM lane) and half of the
//               tile's activation columns each: per group, tcgen05.ld of the
//               accumulator and y += s[n,g] * C_g with packed f32x2 FMAs
//               into 128 register accumulators (registers moved to these
//               warps with setmaxnreg); after the bias unit, the stores
// Every wait is bounded (4 s); a timed-out wait sets the device status word,
// every role runs to its end without waiting, producers let copies in flight
// land, and TMEM is always released.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace afb {
namespace qmmx {

constexpr int BW = 128;                // weight rows per tile (MMA M)
constexpr int BX = 256;                // activation rows per tile (MMA N)
constexpr int BK = 64;                 // K per stage (one group)
constexpr int X_BYTES = BX * BK * 2;   // 32 KB
constexpr int A_BYTES = BW * BK * 2;   // 16 KB
constexpr int THREADS = 512;
constexpr int DEQUANT_THREADS = 128;   // warps 4-7, one weight row each
constexpr int EPILOGUE_THREADS = 256;  // warps 8-15
constexpr int ACC_COLS = 256;          // TMEM columns per accumulator
// Registers: launched at 128 per thread (512 x 128, the whole file); the
// control and dequantising warpgroups give registers back on entering their
// roles and the two epilogue warpgroups take them, room for 128 accumulators
// per epilogue thread.
constexpr int kLaunchRegs = 128, kControlRegs = 40, kDequantRegs = 72, kEpilogueRegs = 200;
static_assert(128 * kControlRegs + 128 * kDequantRegs + 256 * kEpilogueRegs <= THREADS * kLaunchRegs,
              "register split exceeds the launch allocation");

struct Params {
    const uint16_t *s;
    int64_t lds;
    const uint16_t *b;
    int64_t ldb;
    void *y;
    int64_t ldy;
    unsigned *status;
    int M, N, K;
    int G;           // groups along K
    int nbs;         // bias stages per tile (KB3 / 64)
    int m_blocks, tiles;
    int y_bf16;
    int s_vec;       // scale rows 16-byte aligned and G % 8 == 0: eight scales per load
};

// Groups per bias stage: a stage's 64 columns hold three X pieces of each of
// 21 groups (63 columns) and one zero column.
constexpr int BIAS_GROUPS = 21;

// Rings: activation (or X-piece) tiles, the longest-latency loads, get the
// most stages; code tiles are produced in shared memory by the dequantisers
// and need few.
template <int BITS>
struct Cfg {
    static constexpr int XSTAGES = 5;
    static constexpr int ASTAGES = 3;
    static constexpr int PSTAGES = BITS == 4 ? 3 : 2;
    static constexpr int P_ROW = BK * BITS / 8;      // packed bytes per row per stage
    static constexpr int P_BYTES = BW * P_ROW;
    static constexpr int SMEM = 1024 + XSTAGES * X_BYTES + ASTAGES * A_BYTES + PSTAGES * P_BYTES + 512;
    static_assert(SMEM <= 232448, "shared memory per block");
};

// y0,y1 += s * (c0, c1): one packed f32x2 fused multiply-add.
__device__ __forceinline__ void ffma2(float &y0, float &y1, float s, uint32_t c0, uint32_t c1) {
    uint64_t acc = (static_cast<uint64_t>(__float_as_uint(y1)) << 32) | __float_as_uint(y0);
    const uint64_t ss = (static_cast<uint64_t>(__float_as_uint(s)) << 32) | __float_as_uint(s);
    const uint64_t cc = (static_cast<uint64_t>(c1) << 32) | c0;
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(ss), "l"(cc));
    y0 = __uint_as_float(static_cast<uint32_t>(acc));
    y1 = __uint_as_float(static_cast<uint32_t>(acc >> 32));
}

// y += scale * D for the accumulator of the unit with sequence number
// `count` (buffer count & 1): 128 activation columns of weight row i, read
// from TMEM in 16-column pieces, the next piece loading while the current one
// is applied.  The buffer is released to the MMA as soon as the last piece is
// in registers.  Called by every epilogue thread.
__device__ __forceinline__ void apply_unit(float (&y)[BX / 2], float scale, uint32_t count, uint32_t tmem,
                                          uint64_t *accfull, uint64_t *accempty, volatile int *abort,
                                          unsigned *status, int q, int h) {
    const int buf = count & 1;
    mbar_wait(&accfull[buf], (count >> 1) & 1, abort, status);
    tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * ACC_COLS + h * (BX / 2);
    constexpr int PIECES = BX / 32;
    uint32_t ra[16], rb[16];
    tmem_ld_32x32b_x16(base, ra);
#pragma unroll
    for (int c = 0; c < PIECES; c += 2) {
        tmem_wait_ld(ra);
        tmem_ld_32x32b_x16(base + 16 * (c + 1), rb);
#pragma unroll
        for (int j = 0; j < 8; ++j) ffma2(y[16 * c + 2 * j], y[16 * c + 2 * j + 1], scale, ra[2 * j], ra[2 * j + 1]);
        tmem_wait_ld(rb);
        if (c + 2 < PIECES) {
            tmem_ld_32x32b_x16(base + 16 * (c + 2), ra);
        } else {  // every piece is in registers: release the accumulator
            tc_fence_before();
            mbar_arrive(&accempty[buf]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            ffma2(y[16 * (c + 1) + 2 * j], y[16 * (c + 1) + 2 * j + 1], scale, rb[2 * j], rb[2 * j + 1]);
    }
}

// The last unit of a tile (the bias term, scale 1): y += D, then the stores,
// 16 activation rows at a time as each piece of the accumulator arrives.
// y_out[m0 + j][n] for j < lim.
__device__ __forceinline__ void finish_tile(float (&y)[BX / 2], uint32_t count, uint32_t tmem, uint64_t *accfull,
                                            uint64_t *accempty, volatile int *abort, unsigned *status, int q, int h,
                                            const Params &p, int64_t m0, int64_t n) {
    const int buf = count & 1;
    mbar_wait(&accfull[buf], (count >> 1) & 1, abort, status);
    tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * ACC_COLS + h * (BX / 2);
    const int64_t lim = p.M - m0;
    const bool live = n < p.N;
#pragma unroll
    for (int c = 0; c < BX / 32; ++c) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(base + 16 * c, r);
        tmem_wait_ld(r);
        if (c == BX / 32 - 1) {
            tc_fence_before();
            mbar_arrive(&accempty[buf]);
        }
        if (live) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int jj = 16 * c + j;
                const float v = y[jj] + __uint_as_float(r[j]);
                if (jj < lim) {
                    if (p.y_bf16)
                        static_cast<uint16_t *>(p.y)[(m0 + jj) * p.ldy + n] = f32_to_bf16_bits(v);
                    else
                        static_cast<float *>(p.y)[(m0 + jj) * p.ldy + n] = v;
                }
            }
        }
    }
}

template <int BITS>
__global__ void __launch_bounds__(THREADS, 1)
    qmm_exact_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xsmap,
                     const __grid_constant__ CUtensorMap wmap, Params p) {
    using C = Cfg<BITS>;
    constexpr int SX = C::XSTAGES, SA = C::ASTAGES, PS = C::PSTAGES;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char *xs = smem;                                  // SX x 32 KB activation (or X-piece) tiles
    char *as = xs + SX * X_BYTES;                     // SA x 16 KB code (or repeated-bias) tiles
    char *ps = as + SA * A_BYTES;                     // PS packed tiles
    uint64_t *bars = reinterpret_cast<uint64_t *>(ps + PS * C::P_BYTES);
    uint64_t *xfull = bars, *xempty = xfull + SX, *afull = xempty + SX, *aempty = afull + SA;
    uint64_t *pfull = aempty + SA, *pempty = pfull + PS;
    uint64_t *accfull = pempty + PS, *accempty = accfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accempty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < SX; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], 1);
        }
        for (int i = 0; i < SA; ++i) {
            mbar_init(&afull[i], DEQUANT_THREADS);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < PS; ++i) {
            mbar_init(&pfull[i], 1);
            mbar_init(&pempty[i], DEQUANT_THREADS);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accfull[i], 1);
            mbar_init(&accempty[i], EPILOGUE_THREADS);
        }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * ACC_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int G = p.G, SPT = p.G + p.nbs;  // stages per tile: code groups, then bias stages

    if (warp == 0) {  // -------------------------------- activation / X-piece TMA
        regs_release<kControlRegs>();
        if (lane == 0) {
            tma_prefetch_desc(&xmap);
            tma_prefetch_desc(&xsmap);
            int s = 0;
            uint32_t ph = 0, issued = 0, par = 0;
            for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
                const int mb = t % p.m_blocks;
                for (int st = 0; st < SPT; ++st) {
                    if (mbar_wait(&xempty[s], ph ^ 1, abort, p.status) && !*abort) {  // never re-arm after an abort
                        mbar_arrive_expect_tx(&xfull[s], X_BYTES);
                        if (st < G)
                            tma_load_2d(xs + s * X_BYTES, &xmap, &xfull[s], st * BK, mb * BX);
                        else
                            tma_load_2d(xs + s * X_BYTES, &xsmap, &xfull[s], (st - G) * BK, mb * BX);
                        issued |= 1u << s;
                        par = (par & ~(1u << s)) | (ph << s);
                    }
                    if (++s == SX) { s = 0; ph ^= 1; }
                }
            }
            // Let every copy issued land before the CTA can exit.
            for (int i = 0; i < SX; ++i)
                if (issued & (1u << i)) mbar_wait_drain(&xfull[i], (par >> i) & 1u);
        }
        __syncwarp();
    } else if (warp == 2) {  // ------------------------------------ packed TMA
        regs_release<kControlRegs>();
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            int s = 0;
            uint32_t ph = 0, issued = 0, par = 0;
            for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
                const int nb = t / p.m_blocks;
                for (int g = 0; g < G; ++g) {
                    if (mbar_wait(&pempty[s], ph ^ 1, abort, p.status) && !*abort) {
                        mbar_arrive_expect_tx(&pfull[s], C::P_BYTES);
                        tma_load_2d(ps + s * C::P_BYTES, &wmap, &pfull[s], g * (BK * BITS / 32), nb * BW);
                        issued |= 1u << s;
                        par = (par & ~(1u << s)) | (ph << s);
                    }
                    if (++s == PS) { s = 0; ph ^= 1; }
                }
            }
            for (int i = 0; i < PS; ++i)
                if (issued & (1u << i)) mbar_wait_drain(&pfull[i], (par >> i) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {  // ------------------------------------ MMA issuer
        regs_release<kControlRegs>();
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(BW, BX);
            int sx = 0, sa = 0;
            uint32_t xph = 0, aph = 0, uc = 0;
            for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
                for (int u = 0; u <= G; ++u, ++uc) {  // unit G: the bias term
                    const int buf = uc & 1;
                    const uint32_t d_tmem = tmem + buf * ACC_COLS;
                    mbar_wait(&accempty[buf], ((uc >> 1) & 1) ^ 1, abort, p.status);
                    tc_fence_after();
                    const int nst = u < G ? 1 : p.nbs;
                    for (int st = 0; st < nst; ++st) {
                        bool ok = mbar_wait(&xfull[sx], xph, abort, p.status);
                        ok = mbar_wait(&afull[sa], aph, abort, p.status) && ok;
                        tc_fence_after();
                        if (ok) {
                            const uint32_t a0 = smem_u32(as + sa * A_BYTES), b0 = smem_u32(xs + sx * X_BYTES);
#pragma unroll
                            for (int k = 0; k < BK / 16; ++k)
                                umma_bf16_ss(d_tmem, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc,
                                             (st | k) != 0);
                        }
                        umma_commit(&xempty[sx]);
                        umma_commit(&aempty[sa]);
                        if (++sx == SX) { sx = 0; xph ^= 1; }
                        if (++sa == SA) { sa = 0; aph ^= 1; }
                    }
                    umma_commit(&accfull[buf]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 3) {
        regs_release<kControlRegs>();
    } else if (warp < 8) {  // ------------------------------------- dequantisers
        regs_release<kDequantRegs>();
        const int i = tid - 128;  // weight row within the tile
        int s = 0, ps_i = 0;
        uint32_t ph = 0, pph = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
            const int nb = t / p.m_blocks;
            const int64_t n = std::min(static_cast<int64_t>(nb) * BW + i, static_cast<int64_t>(p.N - 1));
            const uint16_t *brow = p.b + n * p.ldb;
            for (int st = 0; st < SPT; ++st) {
                mbar_wait(&aempty[s], ph ^ 1, abort, p.status);
                char *arow = as + s * A_BYTES + i * 128;
                if (st < G) {
                    mbar_wait(&pfull[ps_i], pph, abort, p.status);
                    const char *prow = ps + ps_i * C::P_BYTES + i * C::P_ROW;
#pragma unroll
                    for (int v = 0; v < C::P_ROW / 16; ++v) {
                        const uint4 qv = *reinterpret_cast<const uint4 *>(prow + 16 * v);
                        const uint32_t wv[4] = {qv.x, qv.y, qv.z, qv.w};
                        if constexpr (BITS == 4) {
#pragma unroll
                            for (int j = 0; j < 4; ++j) {  // 16-byte chunk 4v+j holds K = 32v+8j .. +7
                                uint32_t o[4];
                                dec4_nat(wv[j], o);
                                *reinterpret_cast<uint4 *>(arow + (((4 * v + j) ^ (i & 7)) << 4)) =
                                    make_uint4(o[0], o[1], o[2], o[3]);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 2; ++j) {  // chunk 2v+j holds K = 16v+8j .. +7
                                const uint4 o = make_uint4(dec8_pair(wv[2 * j], 0), dec8_pair(wv[2 * j], 2),
                                                           dec8_pair(wv[2 * j + 1], 0), dec8_pair(wv[2 * j + 1], 2));
                                *reinterpret_cast<uint4 *>(arow + (((2 * v + j) ^ (i & 7)) << 4)) = o;
                            }
                        }
                    }
                    // The packed stage is free once its words were read; the
                    // proxy fence orders these reads before the next TMA write.
                    fence_proxy_async_smem();
                    mbar_arrive(&pempty[ps_i]);
                    if (++ps_i == PS) { ps_i = 0; pph ^= 1; }
                } else {
                    // Bias stage jb: columns 3k, 3k+1, 3k+2 carry b[n, 21 jb + k]
                    // (zero past the last group), column 63 zero, matching the
                    // X pieces.  The 21 loads are issued together.
                    const int g0 = (st - G) * BIAS_GROUPS;
                    uint32_t bv[BIAS_GROUPS];
#pragma unroll
                    for (int k = 0; k < BIAS_GROUPS; ++k) bv[k] = g0 + k < G ? brow[g0 + k] : 0u;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int c = 8 * j + 2 * e;
                            const uint32_t v0 = c < 63 ? bv[c / 3] : 0u, v1 = c + 1 < 63 ? bv[(c + 1) / 3] : 0u;
                            o[e] = v0 | (v1 << 16);
                        }
                        *reinterpret_cast<uint4 *>(arow + ((j ^ (i & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&afull[s]);
                if (++s == SA) { s = 0; ph ^= 1; }
            }
        }
    } else {  // ------------------------------------------------------ epilogue
        regs_claim<kEpilogueRegs>();
        const int q = warp & 3;            // TMEM lane quarter this warp may access
        const int h = (warp - 8) >> 2;     // half of the tile's activation columns
        const int i = 32 * q + lane;       // weight row within the tile
        uint32_t count = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
            const int nb = t / p.m_blocks, mb = t - nb * p.m_blocks;
            const int64_t n = static_cast<int64_t>(nb) * BW + i;
            const uint16_t *srow = p.s + (n < p.N ? n : p.N - 1) * p.lds;
            float y[BX / 2];
#pragma unroll
            for (int j = 0; j < BX / 2; ++j) y[j] = 0.0f;
            if (p.s_vec) {
                // Scales eight groups per 16-byte load, the next eight in
                // flight while these are applied.
                uint4 cur = ldg_nc_v4(srow), nxt = G > 8 ? ldg_nc_v4(srow + 8) : cur;
                for (int g = 0; g < G; ++g, ++count) {
                    const int e = g & 7;
                    const uint32_t word = e < 2 ? cur.x : e < 4 ? cur.y : e < 6 ? cur.z : cur.w;
                    const float sc = __uint_as_float((e & 1) ? (word & 0xFFFF0000u) : (word << 16));
                    if (e == 7) {
                        cur = nxt;
                        if (g + 9 < G) nxt = ldg_nc_v4(srow + g + 9);
                    }
                    apply_unit(y, sc, count, tmem, accfull, accempty, abort, p.status, q, h);
                }
            } else {
                // Scales four groups ahead of their use.
                uint16_t s0 = srow[0], s1 = G > 1 ? srow[1] : 0, s2 = G > 2 ? srow[2] : 0, s3 = G > 3 ? srow[3] : 0;
                for (int g = 0; g < G; ++g, ++count) {
                    const float sc = bf16_bits_to_f32(s0);
                    s0 = s1;
                    s1 = s2;
                    s2 = s3;
                    s3 = g + 4 < G ? srow[g + 4] : 0;
                    apply_unit(y, sc, count, tmem, accfull, accempty, abort, p.status, q, h);
                }
            }
            finish_tile(y, count++, tmem, accfull, accempty, abort, p.status, q, h, p,
                        static_cast<int64_t>(mb) * BX + h * (BX / 2), n);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * ACC_COLS);
    }
}

// X[m,g] = sum of the 64 activations of group g (f32, in order), written as
// bf16 pieces hi, mid, lo: hi = bf16(X), mid = bf16(X - hi), lo = bf16(X - hi
// - mid); each difference is exact in f32 and hi + mid + lo == X.  Group g =
// 21 j + k lands at columns 64 j + 3k .. 64 j + 3k + 2 of xs[m, 0..kb3);
// column 64 j + 63 and the slots past the last group are zero.
__global__ void __launch_bounds__(256) xsplit_kernel(const uint16_t *x, int64_t ldx, int M, int G, int kb3,
                                                     uint16_t *xs) {
    const int slots = (kb3 / 64) * BIAS_GROUPS;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(M) * slots) return;
    const int m = static_cast<int>(idx / slots), g = static_cast<int>(idx - int64_t(m) * slots);
    float X = 0.0f;
    if (g < G) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + m * ldx + static_cast<int64_t>(g) * 64);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const uint4 u = __ldg(src + v);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                X += __uint_as_float(w[e] << 16);
                X += __uint_as_float(w[e] & 0xFFFF0000u);
            }
        }
    }
    const uint16_t hi = f32_to_bf16_bits(X);
    const float r1 = X - bf16_bits_to_f32(hi);
    const uint16_t mid = f32_to_bf16_bits(r1);
    const uint16_t lo = f32_to_bf16_bits(r1 - bf16_bits_to_f32(mid));
    const int j = g / BIAS_GROUPS, k = g - j * BIAS_GROUPS;
    uint16_t *dst = xs + static_cast<int64_t>(m) * kb3 + 64 * j + 3 * k;
    dst[0] = hi;
    dst[1] = mid;
    dst[2] = lo;
    if (k == 0) dst[63] = 0;
}

}  // namespace qmmx

namespace {
constexpr size_t kXsOffset = (kPartialOffset + 1023) & ~size_t(1023);
int64_t kb3_of(int64_t K) { return 64 * ((K / 64 + qmmx::BIAS_GROUPS - 1) / qmmx::BIAS_GROUPS); }
std::atomic<int64_t> g_slice_cap{0};
}  // namespace

void qmm_exact_set_slice_cap(int64_t rows) { g_slice_cap.store(rows); }

size_t qmm_exact_min_workspace(const QmmArgs &a) { return kXsOffset + size_t(qmmx::BX) * kb3_of(a.K) * 2; }

bool qmm_exact_supported(const QmmArgs &a, const char **why) {
    auto no = [&](const char *r) { if (why) *why = r; return false; };
    if (a.bits != 4 && a.bits != 8) return no("qmm_exact: bits must be 4 or 8");
    if (a.group != 64) return no("qmm_exact: group_size must be 64");
    if (!a.x_bf16 || !a.p_bf16) return no("qmm_exact: activations and parameters must be bf16");
    if (a.M < 64) return no("qmm_exact: M < 64");
    if (a.K % 64) return no("qmm_exact: K must be a multiple of 64");
    if (a.x.col_stride != 1 || a.w.col_stride != 1 || a.s.col_stride != 1 || a.b.col_stride != 1)
        return no("qmm_exact: inputs need unit column stride");
    auto al = [](const void *p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    if (!al(a.x.ptr, 16) || (a.x.row_stride * 2) % 16) return no("qmm_exact: x rows must be 16-byte aligned");
    if (!al(a.w.ptr, 16) || (a.w.row_stride * 4) % 16) return no("qmm_exact: packed rows must be 16-byte aligned");
    if (a.M >= (int64_t(1) << 31) || a.N >= (int64_t(1) << 31) || a.K >= (int64_t(1) << 24))
        return no("qmm_exact: size beyond 32-bit indexing");
    return true;
}

template <int BITS>
static cudaError_t launch_exact_bits(const QmmArgs &a, void *workspace, size_t workspace_bytes, cudaStream_t stream) {
    using C = qmmx::Cfg<BITS>;
    const int64_t G = a.K / 64, kb3 = kb3_of(a.K);
    if (workspace_bytes < qmm_exact_min_workspace(a)) return cudaErrorInvalidValue;
    // Rows of the X-piece array that fit the workspace, in whole tiles.
    const int64_t fit = static_cast<int64_t>((workspace_bytes - kXsOffset) / (size_t(kb3) * 2));
    int64_t slice_rows = (fit / qmmx::BX) * qmmx::BX;
    const int64_t cap = (g_slice_cap.load() / qmmx::BX) * qmmx::BX;
    if (cap > 0) slice_rows = std::min(slice_rows, cap);
    slice_rows = std::min(slice_rows, a.M);
    uint16_t *xs = reinterpret_cast<uint16_t *>(static_cast<char *>(workspace) + kXsOffset);
    auto kern = qmmx::qmm_exact_kernel<BITS>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(kern), C::SMEM);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const CUtensorMap *wm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w.ptr, a.K * BITS / 32, a.N,
                                                 a.w.row_stride * 4, qmmx::BK * BITS / 32, qmmx::BW,
                                                 CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!wm) return cudaErrorInvalidValue;
    for (int64_t m0 = 0; m0 < a.M; m0 += slice_rows) {
        const int64_t rows = std::min(slice_rows, a.M - m0);
        const uint16_t *x = reinterpret_cast<const uint16_t *>(a.x.ptr) + m0 * a.x.row_stride;
        const CUtensorMap *xm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, a.K, rows,
                                                     a.x.row_stride * 2, qmmx::BK, qmmx::BX,
                                                     CU_TENSOR_MAP_SWIZZLE_128B);
        const CUtensorMap *xsm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xs, kb3, rows, kb3 * 2,
                                                      qmmx::BK, qmmx::BX, CU_TENSOR_MAP_SWIZZLE_128B);
        if (!xm || !xsm) return cudaErrorInvalidValue;
        const int64_t items = rows * (kb3 / 64) * qmmx::BIAS_GROUPS;
        qmmx::xsplit_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(
            x, a.x.row_stride, static_cast<int>(rows), static_cast<int>(G), static_cast<int>(kb3), xs);
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        qmmx::Params p{};
        p.s = static_cast<const uint16_t *>(a.s.ptr);
        p.lds = a.s.row_stride;
        p.b = static_cast<const uint16_t *>(a.b.ptr);
        p.ldb = a.b.row_stride;
        p.y = static_cast<char *>(a.y) + m0 * a.ldy * (a.y_bf16 ? 2 : 4);
        p.ldy = a.ldy;
        p.status = static_cast<unsigned *>(workspace);
        p.M = static_cast<int>(rows);
        p.N = static_cast<int>(a.N);
        p.K = static_cast<int>(a.K);
        p.G = static_cast<int>(G);
        p.nbs = static_cast<int>(kb3 / 64);
        p.m_blocks = static_cast<int>((rows + qmmx::BX - 1) / qmmx::BX);
        const int n_blocks = static_cast<int>((a.N + qmmx::BW - 1) / qmmx::BW);
        p.tiles = p.m_blocks * n_blocks;
        p.y_bf16 = a.y_bf16;
        p.s_vec = (reinterpret_cast<uintptr_t>(a.s.ptr) % 16 == 0) && (a.s.row_stride % 8 == 0) && (G % 8 == 0);
        const int grid = std::min(p.tiles, sms);
        kern<<<grid, qmmx::THREADS, C::SMEM, stream>>>(*xm, *xsm, *wm, p);
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_qmm_exact(const QmmArgs &a, void *workspace, size_t workspace_bytes, cudaStream_t stream) {
    return a.bits == 4 ? launch_exact_bits<4>(a, workspace, workspace_bytes, stream)
                       : launch_exact_bits<8>(a, workspace, workspace_bytes, stream);
}

}  // namespace afb
