// Decode qmv for sm_100a: y[M,N] = x[M,K] . decode(W)[N,K]^T for M <= 16,
// 4- or 8-bit codes packed little-endian into u32 along K, group 64, bf16
// activations / scales / biases, f32 accumulation (the layout and formula of
// docs/core/quantized-inference.md:45-67).
//
// Why tensor cores at M <= 16: at the HBM rate of a B200 (~6.5 TB/s) a 4-bit
// weight stream delivers ~11.6e12 weights/s; decoding each weight to a float
// and multiplying it on the CUDA cores costs ~3 lane-ops, which is as much as
// the 148 SMs can issue.  So each warp decodes its packed words in registers
// straight into the A fragments of m16n8k16 bf16 MMAs (no shared-memory round
// trip for the weights), with the activations as the B operand.
//
// Exact codes, per-group affine in f32: the MMA multiplies the *integer codes*
// q (exact in bf16) by x, giving C_g = sum_{k in g} x*q in f32.  The affine
// decode is applied per group of 64 outside the tensor core:
//     y += s[n,g] * C_g + b[n,g] * X_g,   X_g = sum_{k in g} x[k]   (f32)
// which is sum_k x*(s*q+b) up to reassociation; weights are never rounded to
// bf16 (quantized-inference.md:119-121).  Numerical class: reassociated.
//
// Work decomposition: 16-row N tiles (one m16 MMA tile), one warp per tile.
// K is cut into `splits` ranges; a CTA stages its range of x in shared memory
// once (permuted into MMA-fragment order for 4-bit) together with X_g, then
// its 8 warps stream their tiles' packed weights with 8/16-byte read-only
// loads, software-pipelined over 256-K blocks.  With splits > 1 each warp
// writes an f32 partial; the warp that completes a tile last (per-tile
// arrival counter) sums the partials in split order and stores y, so results
// do not depend on scheduling, and it resets the counter for the next launch.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace afb {
namespace qmv {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int GROUP = 64;
constexpr int BG = 4;             // groups per pipeline block
constexpr int BK = BG * GROUP;    // K per pipeline block
constexpr int XS_PAD = 8;         // bf16 elements of padding per staged x row

struct Params {
    const uint16_t *x;
    int64_t ldx;
    const uint32_t *w;
    int64_t ldw;
    const uint16_t *s;
    int64_t lds;
    const uint16_t *b;
    int64_t ldb;
    void *y;
    int64_t ldy;
    float *partial;
    unsigned *counters;
    int M, N;
    int splits;
    int blocks_per_split;
    int tiles;
    int y_bf16;
};

template <int BITS>
struct Blk;
template <>
struct Blk<4> {
    uint2 w[2][BG];  // rows g and g+8: two words (16 codes) per group
    uint2 s[2], b[2];
};
template <>
struct Blk<8> {
    uint4 w[2][BG];  // rows g and g+8: four words (16 codes) per group
    uint2 s[2], b[2];
};

template <int BITS>
__device__ __forceinline__ void load_block(Blk<BITS> &B, const Params &p, int64_t row0, int64_t row1, int G0, int t) {
    constexpr int WPG = 2 * BITS;  // u32 words per row per group of 64
    constexpr int TW = WPG / 4;    // words per thread per row per group
    const uint32_t *r0 = p.w + row0 * p.ldw + static_cast<int64_t>(G0) * WPG + t * TW;
    const uint32_t *r1 = p.w + row1 * p.ldw + static_cast<int64_t>(G0) * WPG + t * TW;
#pragma unroll
    for (int gi = 0; gi < BG; ++gi) {
        if constexpr (BITS == 4) {
            B.w[0][gi] = ldg_stream_v2(r0 + gi * WPG);
            B.w[1][gi] = ldg_stream_v2(r1 + gi * WPG);
        } else {
            B.w[0][gi] = ldg_stream_v4(r0 + gi * WPG);
            B.w[1][gi] = ldg_stream_v4(r1 + gi * WPG);
        }
    }
    B.s[0] = ldg_nc_v2(p.s + row0 * p.lds + G0);
    B.s[1] = ldg_nc_v2(p.s + row1 * p.lds + G0);
    B.b[0] = ldg_nc_v2(p.b + row0 * p.ldb + G0);
    B.b[1] = ldg_nc_v2(p.b + row1 * p.ldb + G0);
}

// Codes p and p+4 of a 4-bit word as an exact bf16 pair (128+q, then -128).
__device__ __forceinline__ uint32_t dec4(uint32_t w, int p) {
    return bf16x2_sub(lop3_and_or(w >> (4 * p), 0x000F000Fu, 0x43004300u), 0x43004300u);
}
// Bytes i and i+1 of an 8-bit word as an exact bf16 pair (via 2^23 + q in f32).
__device__ __forceinline__ uint32_t dec8(uint32_t w, int i) {
    float f0 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i)) - 8388608.0f;
    float f1 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i + 1)) - 8388608.0f;
    return pack_bf16x2(f0, f1);
}

__device__ __forceinline__ float bf16_lane(uint2 v, int i) {
    uint32_t word = (i < 2) ? v.x : v.y;
    return __uint_as_float((i & 1) ? (word & 0xFFFF0000u) : (word << 16));
}

template <int BITS, int MT>
__device__ __forceinline__ void compute_block(const Blk<BITS> &B, float (&acc)[MT][4], const char *xs, int xs_rs,
                                              const float *xg, int Gl0, int g, int t, int M) {
#pragma unroll
    for (int gi = 0; gi < BG; ++gi) {
        const int Gl = Gl0 + gi;
        uint32_t xf[MT][8];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int m = g + 8 * mt;
            if (m < M) {
                const char *src = xs + m * xs_rs + (Gl * GROUP + 16 * t) * 2;
                uint4 v0 = *reinterpret_cast<const uint4 *>(src);
                uint4 v1 = *reinterpret_cast<const uint4 *>(src + 16);
                xf[mt][0] = v0.x; xf[mt][1] = v0.y; xf[mt][2] = v0.z; xf[mt][3] = v0.w;
                xf[mt][4] = v1.x; xf[mt][5] = v1.y; xf[mt][6] = v1.z; xf[mt][7] = v1.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) xf[mt][i] = 0u;
            }
        }
        float c[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) c[mt][0] = c[mt][1] = c[mt][2] = c[mt][3] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t a[4];
            uint32_t b0[MT], b1[MT];
            if constexpr (BITS == 4) {
                const uint32_t w0 = (j < 2) ? B.w[0][gi].x : B.w[0][gi].y;
                const uint32_t w1 = (j < 2) ? B.w[1][gi].x : B.w[1][gi].y;
                const int p0 = 2 * (j & 1);
                a[0] = dec4(w0, p0);
                a[1] = dec4(w1, p0);
                a[2] = dec4(w0, p0 + 1);
                a[3] = dec4(w1, p0 + 1);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    b0[mt] = xf[mt][4 * (j >> 1) + p0];
                    b1[mt] = xf[mt][4 * (j >> 1) + p0 + 1];
                }
            } else {
                const uint32_t w0 = (j == 0) ? B.w[0][gi].x : (j == 1) ? B.w[0][gi].y : (j == 2) ? B.w[0][gi].z : B.w[0][gi].w;
                const uint32_t w1 = (j == 0) ? B.w[1][gi].x : (j == 1) ? B.w[1][gi].y : (j == 2) ? B.w[1][gi].z : B.w[1][gi].w;
                a[0] = dec8(w0, 0);
                a[1] = dec8(w1, 0);
                a[2] = dec8(w0, 2);
                a[3] = dec8(w1, 2);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    b0[mt] = xf[mt][2 * j];
                    b1[mt] = xf[mt][2 * j + 1];
                }
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) mma_bf16_16816(c[mt], a, b0[mt], b1[mt], c[mt]);
        }
        const float s0 = bf16_lane(B.s[0], gi), s1 = bf16_lane(B.s[1], gi);
        const float q0 = bf16_lane(B.b[0], gi), q1 = bf16_lane(B.b[1], gi);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const float2 X = *reinterpret_cast<const float2 *>(xg + Gl * 16 + 2 * t + 8 * mt);
            acc[mt][0] = fmaf(s0, c[mt][0], fmaf(q0, X.x, acc[mt][0]));
            acc[mt][1] = fmaf(s0, c[mt][1], fmaf(q0, X.y, acc[mt][1]));
            acc[mt][2] = fmaf(s1, c[mt][2], fmaf(q1, X.x, acc[mt][2]));
            acc[mt][3] = fmaf(s1, c[mt][3], fmaf(q1, X.y, acc[mt][3]));
        }
    }
}

__device__ __forceinline__ void store_out(const Params &p, int m, int64_t n, float v) {
    if (p.y_bf16)
        static_cast<uint16_t *>(p.y)[m * p.ldy + n] = f32_to_bf16_bits(v);
    else
        static_cast<float *>(p.y)[m * p.ldy + n] = v;
}

template <int MT>
__device__ __forceinline__ void tile_epilogue(const Params &p, float (&acc)[MT][4], int tile, int split, int g, int t,
                                              int lane) {
    const int64_t n0 = static_cast<int64_t>(tile) * 16;
    if (p.splits == 1) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = 2 * t + 8 * mt + (i & 1);
                const int64_t n = n0 + g + 8 * (i >> 1);
                if (m < p.M && n < p.N) store_out(p, m, n, acc[mt][i]);
            }
        return;
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = 2 * t + 8 * mt + (i & 1);
            const int64_t n = n0 + g + 8 * (i >> 1);
            if (m < p.M && n < p.N) p.partial[(static_cast<int64_t>(split) * p.M + m) * p.N + n] = acc[mt][i];
        }
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(&p.counters[tile], 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != static_cast<unsigned>(p.splits - 1)) return;
    __threadfence();
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = 2 * t + 8 * mt + (i & 1);
            const int64_t n = n0 + g + 8 * (i >> 1);
            if (m < p.M && n < p.N) {
                float sum = 0.0f;
                for (int sp = 0; sp < p.splits; ++sp) sum += __ldcg(&p.partial[(static_cast<int64_t>(sp) * p.M + m) * p.N + n]);
                store_out(p, m, n, sum);
            }
        }
    __syncwarp();
    if (lane == 0) atomicExch(&p.counters[tile], 0u);
}

template <int BITS, int MT, int STAGES>
__global__ void __launch_bounds__(THREADS, 1) qmv_kernel(Params p) {
    extern __shared__ __align__(16) char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int split = blockIdx.y;
    const int nb = p.blocks_per_split;
    const int Ks = nb * BK;
    const int Gs = Ks / GROUP;
    const int64_t k0 = static_cast<int64_t>(split) * Ks;
    const int xs_rs = (Ks + XS_PAD) * 2;
    char *xs = smem;
    float *xg = reinterpret_cast<float *>(smem + static_cast<size_t>(p.M) * xs_rs);

    // Stage x[:, k0:k0+Ks) (4-bit: each 8-element word permuted to
    // [x0 x4 x1 x5 x2 x6 x3 x7] so that B fragments match the nibble pairs
    // dec4 produces) and the per-group sums X_g.
    for (int i = tid; i < Gs * 16; i += THREADS) xg[i] = 0.0f;
    __syncthreads();
    const int cpr = Ks / 8;  // 16-byte chunks per row
    const int total = p.M * cpr;
    for (int base = 0; base < total; base += THREADS) {
        const int c = base + tid;
        const bool valid = c < total;
        const int m = valid ? c / cpr : 0, kc = valid ? c % cpr : 0;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) v = ldg_nc_v4(p.x + m * p.ldx + k0 + kc * 8);
        float sum = bf16_bits_to_f32(v.x & 0xFFFF) + bf16_bits_to_f32(v.x >> 16) + bf16_bits_to_f32(v.y & 0xFFFF) +
                    bf16_bits_to_f32(v.y >> 16) + bf16_bits_to_f32(v.z & 0xFFFF) + bf16_bits_to_f32(v.z >> 16) +
                    bf16_bits_to_f32(v.w & 0xFFFF) + bf16_bits_to_f32(v.w >> 16);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (valid) {
            if constexpr (BITS == 4) {
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
    __syncthreads();

    const int stride = gridDim.x * WARPS;
    const int tile0 = blockIdx.x * WARPS + warp;
    const int my_tiles = tile0 < p.tiles ? (p.tiles - 1 - tile0) / stride + 1 : 0;
    const int total_steps = my_tiles * nb;
    if (total_steps == 0) return;

    const int gbase = split * nb * BG;  // first absolute group of this split
    auto rows_of = [&](int step, int64_t &r0, int64_t &r1, int &blk, int &tile) {
        const int ti = step / nb;
        blk = step - ti * nb;
        tile = tile0 + ti * stride;
        const int64_t n0 = static_cast<int64_t>(tile) * 16;
        r0 = min(n0 + g, static_cast<int64_t>(p.N - 1));
        r1 = min(n0 + g + 8, static_cast<int64_t>(p.N - 1));
    };

    Blk<BITS> buf[STAGES];
#pragma unroll
    for (int st = 0; st < STAGES; ++st) {
        if (st < total_steps) {
            int64_t r0, r1;
            int blk, tile;
            rows_of(st, r0, r1, blk, tile);
            load_block<BITS>(buf[st], p, r0, r1, gbase + blk * BG, t);
        }
    }
    float acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;

    for (int step = 0; step < total_steps; step += STAGES) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) {
            const int s = step + st;
            if (s < total_steps) {
                int64_t r0, r1;
                int blk, tile;
                rows_of(s, r0, r1, blk, tile);
                compute_block<BITS, MT>(buf[st], acc, xs, xs_rs, xg, blk * BG, g, t, p.M);
                if (s + STAGES < total_steps) {
                    int64_t q0, q1;
                    int qb, qt;
                    rows_of(s + STAGES, q0, q1, qb, qt);
                    load_block<BITS>(buf[st], p, q0, q1, gbase + qb * BG, t);
                }
                if (blk == nb - 1) {
                    tile_epilogue<MT>(p, acc, tile, split, g, t, lane);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;
                }
            }
        }
    }
}

template <int BITS, int MT, int STAGES>
cudaError_t launch_cfg(const Params &p, const QmvPlan &plan, cudaStream_t stream) {
    auto kern = qmv_kernel<BITS, MT, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, plan.smem_bytes);
    if (e != cudaSuccess) return e;
    // Size the grid to the resident CTAs (registers and shared memory both
    // limit it), so every split's CTAs run in one wave and warps loop over tiles.
    int per_sm = 1, dev = 0, sms = 148;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, THREADS, plan.smem_bytes)) != cudaSuccess)
        return e;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const int64_t ctas_needed = (p.tiles + WARPS - 1) / WARPS;
    const int64_t slots = static_cast<int64_t>(sms) * (per_sm > 0 ? per_sm : 1);
    const int grid_n = static_cast<int>(std::max<int64_t>(1, std::min(ctas_needed, (slots + plan.splits - 1) / plan.splits)));
    dim3 grid(grid_n, plan.splits);
    kern<<<grid, THREADS, plan.smem_bytes, stream>>>(p);
    count_launch();
    return cudaGetLastError();
}

}  // namespace qmv

bool qmv_supported(const QmmArgs &a, const char **why) {
    auto no = [&](const char *r) { if (why) *why = r; return false; };
    if (a.bits != 4 && a.bits != 8) return no("qmv: bits must be 4 or 8");
    if (a.group != 64) return no("qmv: group_size must be 64");
    if (!a.x_bf16 || !a.p_bf16) return no("qmv: activations and parameters must be bf16");
    if (a.M > 16) return no("qmv: M > 16");
    if (a.K % qmv::BK) return no("qmv: K must be a multiple of 256");
    if (a.x.col_stride != 1 || a.w.col_stride != 1 || a.s.col_stride != 1 || a.b.col_stride != 1)
        return no("qmv: inputs need unit column stride");
    auto al = [](const void *p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    if (!al(a.x.ptr, 16) || a.x.row_stride % 8) return no("qmv: x rows must be 16-byte aligned");
    const int wal = a.bits == 8 ? 16 : 8;
    if (!al(a.w.ptr, wal) || (a.w.row_stride * 4) % wal) return no("qmv: packed rows misaligned");
    if (!al(a.s.ptr, 8) || !al(a.b.ptr, 8) || a.s.row_stride % 4 || a.b.row_stride % 4)
        return no("qmv: parameter rows must be 8-byte aligned");
    if (a.N >= (int64_t(1) << 31) / 16 || a.K >= (int64_t(1) << 30)) return no("qmv: size beyond 32-bit tile indexing");
    return true;
}

static int qmv_smem(const QmmArgs &a, int splits) {
    const int64_t Ks = a.K / splits;
    return static_cast<int>(a.M * (Ks + qmv::XS_PAD) * 2 + (Ks / qmv::GROUP) * 16 * 4);
}

QmvPlan qmv_plan(const QmmArgs &a, int num_sms, size_t workspace_bytes) {
    const int nblk = static_cast<int>(a.K / qmv::BK);
    const int64_t tiles = (a.N + 15) / 16;
    const int smem_cap = 100 * 1024;
    const int64_t target = static_cast<int64_t>(num_sms) * 12;  // warps wanted in flight
    auto ws_ok = [&](int s) {
        return s == 1 || static_cast<size_t>(s) * a.M * a.N * 4 + tiles * 4 + 256 <= workspace_bytes;
    };
    int chosen = 0;
    for (int s = 1; s <= nblk; ++s) {
        if (nblk % s || qmv_smem(a, s) > smem_cap || !ws_ok(s)) continue;
        chosen = s;
        if (tiles * s >= target && nblk / s >= 2) break;
        if (tiles * s >= target) break;
    }
    if (chosen == 0) {  // smallest split that fits shared memory, ignoring parallelism
        for (int s = 1; s <= nblk; ++s)
            if (nblk % s == 0 && qmv_smem(a, s) <= 220 * 1024 && ws_ok(s)) { chosen = s; break; }
    }
    QmvPlan p{};
    p.splits = chosen > 0 ? chosen : 1;
    p.blocks_per_split = nblk / p.splits;
    p.smem_bytes = qmv_smem(a, p.splits);
    const int per_sm = std::max(1, std::min(2, (220 * 1024) / std::max(1, p.smem_bytes)));
    const int64_t ctas_needed = (tiles + qmv::WARPS - 1) / qmv::WARPS;
    const int64_t slots = static_cast<int64_t>(num_sms) * per_sm;
    p.grid_n = static_cast<int>(std::max<int64_t>(1, std::min(ctas_needed, (slots + p.splits - 1) / p.splits)));
    return p;
}

size_t qmv_workspace_bytes(const QmmArgs &a, const QmvPlan &p) {
    if (p.splits <= 1) return 0;
    const int64_t tiles = (a.N + 15) / 16;
    return static_cast<size_t>(p.splits) * a.M * a.N * 4 + static_cast<size_t>(tiles) * 4 + 256;
}

cudaError_t launch_qmv(const QmmArgs &a, const QmvPlan &plan, void *workspace, cudaStream_t stream) {
    qmv::Params p{};
    p.x = static_cast<const uint16_t *>(a.x.ptr);
    p.ldx = a.x.row_stride;
    p.w = static_cast<const uint32_t *>(a.w.ptr);
    p.ldw = a.w.row_stride;
    p.s = static_cast<const uint16_t *>(a.s.ptr);
    p.lds = a.s.row_stride;
    p.b = static_cast<const uint16_t *>(a.b.ptr);
    p.ldb = a.b.row_stride;
    p.y = a.y;
    p.ldy = a.ldy;
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(a.N);
    p.splits = plan.splits;
    p.blocks_per_split = plan.blocks_per_split;
    p.tiles = static_cast<int>((a.N + 15) / 16);
    p.y_bf16 = a.y_bf16;
    if (plan.splits > 1) {
        // Workspace layout: [tiles] arrival counters (kept at zero between
        // launches), then [splits][M][N] f32 partials at a 256-byte boundary.
        p.counters = static_cast<unsigned *>(workspace);
        size_t off = ((static_cast<size_t>(p.tiles) * 4 + 255) / 256) * 256;
        p.partial = reinterpret_cast<float *>(static_cast<char *>(workspace) + off);
    }
    const bool mt2 = a.M > 8;
    if (a.bits == 4)
        return mt2 ? qmv::launch_cfg<4, 2, 3>(p, plan, stream) : qmv::launch_cfg<4, 1, 3>(p, plan, stream);
    return mt2 ? qmv::launch_cfg<8, 2, 2>(p, plan, stream) : qmv::launch_cfg<8, 1, 2>(p, plan, stream);
}

}  // namespace afb
