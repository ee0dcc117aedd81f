// Prefill qmm for sm_100a on 5th-generation tensor cores (tcgen05 + TMEM):
// y[M,N] = x[M,K] . decode(W)[N,K]^T for large M, 4/8-bit codes, group 64,
// bf16 x / scales / biases, f32 accumulation in TMEM.
//
// Tile: 128 weight rows x 256 activation rows x 64 K per stage.  The
// dequantised weight tile is the MMA's A operand (M = 128) and the
// activation tile its B operand (N = 256), so each decoded weight feeds 256
// activation rows and the CUDA-core decode work per MAC is halved compared
// with decoding a 256-row weight tile.  D[n, m] accumulates in TMEM
// (128 lanes x 256 f32 columns), double-buffered so the epilogue of one tile
// overlaps the MMAs of the next.
//
// Warp roles (352 threads, one persistent CTA per SM):
//   warp 0      TMA producer of activation tiles (128-byte swizzle)
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warp 2      TMA producer of packed-weight tiles
//   warps 3-6   dequantisers: packed words -> bf16 w = fma(q, s, b) in the
//               UMMA K-major 128-byte-swizzle layout, then
//               fence.proxy.async so the tensor core sees the writes; the
//               packed stage is released (after another proxy fence) only
//               once its words were decoded
//   warps 7-10  epilogue: tcgen05.ld of the accumulator, f32/bf16 stores
// Every wait is bounded (4 s); a timed-out wait sets the device status word
// and lets all roles run to the end so TMEM is always released.
//
// Numerics: each decoded weight is rounded once to bf16 (fma.rn of the exact
// s*q+b); products and sums are f32.  Relative error per weight <= 2^-9, so
// this kernel is classified `approximate` and is selected for bf16 results
// or numericalPolicy 'approximate' only.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace afb {
namespace qmmtc {

constexpr int BW = 128;   // weight rows per tile (MMA M)
constexpr int BX = 256;   // activation rows per tile (MMA N)
constexpr int BK = 64;    // K per stage (one group)
constexpr int X_BYTES = BX * BK * 2;   // 32 KB
constexpr int A_BYTES = BW * BK * 2;   // 16 KB
constexpr int THREADS = 352;
constexpr int ACC_COLS = 256;

struct Params {
    const uint16_t *s;
    int64_t lds;
    const uint16_t *b;
    int64_t ldb;
    void *y;
    int64_t ldy;
    unsigned *status;
    int M, N, K;
    int m_blocks, n_blocks, tiles;
    int y_bf16;
};

template <int BITS>
struct Cfg {
    static constexpr int STAGES = BITS == 4 ? 4 : 3;
    static constexpr int PSTAGES = 4;
    static constexpr int P_ROW = BK * BITS / 8;      // packed bytes per row per stage
    static constexpr int P_BYTES = BW * P_ROW;
    static constexpr int SMEM = 1024 + STAGES * (X_BYTES + A_BYTES) + PSTAGES * P_BYTES + 512;
};

__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int BITS>
__global__ void __launch_bounds__(THREADS, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap, Params p) {
    using C = Cfg<BITS>;
    constexpr int S = C::STAGES, PS = C::PSTAGES;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char *xs = smem;                                  // S x 32 KB activation tiles
    char *as = xs + S * X_BYTES;                      // S x 16 KB decoded weight tiles
    char *ps = as + S * A_BYTES;                      // PS packed tiles
    uint64_t *bars = reinterpret_cast<uint64_t *>(ps + PS * C::P_BYTES);
    uint64_t *xfull = bars, *afull = xfull + S, *sempty = afull + S;
    uint64_t *pfull = sempty + S, *pempty = pfull + PS;
    uint64_t *accfull = pempty + PS, *accempty = accfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accempty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&afull[i], 128);
            mbar_init(&sempty[i], 1);
        }
        for (int i = 0; i < PS; ++i) {
            mbar_init(&pfull[i], 1);
            mbar_init(&pempty[i], 128);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accfull[i], 1);
            mbar_init(&accempty[i], 128);
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
    const int KB = p.K / BK;

    if (warp == 0) {  // ------------------------------------------ activation TMA
        if (lane == 0) {
            tma_prefetch_desc(&xmap);
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
                const int mb = t % p.m_blocks;
                for (int kb = 0; kb < KB; ++kb) {
                    if (mbar_wait(&sempty[s], ph ^ 1, abort, p.status) && !*abort) {  // never re-arm after an abort
                        mbar_arrive_expect_tx(&xfull[s], X_BYTES);
                        tma_load_2d(xs + s * X_BYTES, &xmap, &xfull[s], kb * BK, mb * BX);
                    }
                    if (++s == S) { s = 0; ph ^= 1; }
                }
            }
        }
        __syncwarp();  // reconverge before the CTA-wide barrier at the end
    } else if (warp == 2) {  // ------------------------------------ packed TMA
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
                const int nb = t / p.m_blocks;
                for (int kb = 0; kb < KB; ++kb) {
                    if (mbar_wait(&pempty[s], ph ^ 1, abort, p.status) && !*abort) {
                        mbar_arrive_expect_tx(&pfull[s], C::P_BYTES);
                        tma_load_2d(ps + s * C::P_BYTES, &wmap, &pfull[s], kb * (BK * BITS / 32), nb * BW);
                    }
                    if (++s == PS) { s = 0; ph ^= 1; }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {  // ------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(BW, BX);
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++it) {
                const int buf = it & 1;
                const uint32_t d_tmem = tmem + buf * ACC_COLS;
                mbar_wait(&accempty[buf], ((it >> 1) & 1) ^ 1, abort, p.status);
                tc_fence_after();
                for (int kb = 0; kb < KB; ++kb) {
                    bool ok = mbar_wait(&xfull[s], ph, abort, p.status);
                    ok = mbar_wait(&afull[s], ph, abort, p.status) && ok;
                    tc_fence_after();
                    if (ok) {
                        const uint32_t a0 = smem_u32(as + s * A_BYTES), b0 = smem_u32(xs + s * X_BYTES);
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)
                            umma_bf16_ss(d_tmem, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc,
                                         (kb | k) != 0);
                    }
                    umma_commit(&sempty[s]);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                umma_commit(&accfull[buf]);
            }
        }
        __syncwarp();
    } else if (warp < 7) {  // ------------------------------------- dequantisers
        const int i = tid - 96;  // weight row within the tile
        int s = 0, ps_i = 0;
        uint32_t ph = 0, pph = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
            const int nb = t / p.m_blocks;
            const int64_t row = min(static_cast<int64_t>(nb) * BW + i, static_cast<int64_t>(p.N - 1));
            const uint16_t *srow = p.s + row * p.lds, *brow = p.b + row * p.ldb;
            uint4 sc = ldg_nc_v4(srow), bc = ldg_nc_v4(brow);  // groups 0..7
            uint4 sn = sc, bn = bc;
            for (int kb = 0; kb < KB; ++kb) {
                if ((kb & 7) == 0) {
                    if (kb) { sc = sn; bc = bn; }
                    if (kb + 8 < KB) {
                        sn = ldg_nc_v4(srow + kb + 8);
                        bn = ldg_nc_v4(brow + kb + 8);
                    }
                }
                const int gi = kb & 7;
                const uint32_t sw = (gi < 2 ? sc.x : gi < 4 ? sc.y : gi < 6 ? sc.z : sc.w);
                const uint32_t bw = (gi < 2 ? bc.x : gi < 4 ? bc.y : gi < 6 ? bc.z : bc.w);
                const uint32_t s2 = (gi & 1) ? ((sw >> 16) | (sw & 0xFFFF0000u)) : ((sw & 0xFFFFu) | (sw << 16));
                const uint32_t b2 = (gi & 1) ? ((bw >> 16) | (bw & 0xFFFF0000u)) : ((bw & 0xFFFFu) | (bw << 16));
                mbar_wait(&sempty[s], ph ^ 1, abort, p.status);
                mbar_wait(&pfull[ps_i], pph, abort, p.status);
                const char *prow = ps + ps_i * C::P_BYTES + i * C::P_ROW;
                uint32_t wv[BK * BITS / 32];
#pragma unroll
                for (int v = 0; v < BK * BITS / 128; ++v) {
                    const uint4 q = *reinterpret_cast<const uint4 *>(prow + 16 * v);
                    wv[4 * v] = q.x; wv[4 * v + 1] = q.y; wv[4 * v + 2] = q.z; wv[4 * v + 3] = q.w;
                }
                char *arow = as + s * A_BYTES + i * 128;
#pragma unroll
                for (int j = 0; j < 8; ++j) {  // 16-byte chunk j holds K = 8j..8j+7
                    uint32_t o[4];
                    if constexpr (BITS == 4) {
                        dec4_nat(wv[j], o);
                    } else {
                        o[0] = dec8_pair(wv[2 * j], 0);
                        o[1] = dec8_pair(wv[2 * j], 2);
                        o[2] = dec8_pair(wv[2 * j + 1], 0);
                        o[3] = dec8_pair(wv[2 * j + 1], 2);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[e] = bf16x2_fma(o[e], s2, b2);
                    *reinterpret_cast<uint4 *>(arow + ((j ^ (i & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
                // Release the packed stage only after its words were consumed,
                // with a proxy fence: the next TMA write (async proxy) must be
                // ordered after these generic-proxy reads.
                fence_proxy_async_smem();
                mbar_arrive(&pempty[ps_i]);
                if (++ps_i == PS) { ps_i = 0; pph ^= 1; }
                fence_proxy_async_smem();
                mbar_arrive(&afull[s]);
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else {  // ------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int it = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++it) {
            const int buf = it & 1;
            const int mb = t % p.m_blocks, nb = t / p.m_blocks;
            mbar_wait(&accfull[buf], (it >> 1) & 1, abort, p.status);
            tc_fence_after();
            const int64_t n = static_cast<int64_t>(nb) * BW + 32 * q + lane;
            const uint32_t base = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * ACC_COLS;
#pragma unroll 1
            for (int c = 0; c < ACC_COLS / 16; ++c) {
                uint32_t r[16];
                tmem_ld_32x32b_x16(base + c * 16, r);
                tmem_wait_ld(r);
                const int m0 = mb * BX + c * 16;
                if (n < p.N) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int m = m0 + j;
                        if (m < p.M) {
                            if (p.y_bf16)
                                static_cast<uint16_t *>(p.y)[m * p.ldy + n] = f32_to_bf16_bits(__uint_as_float(r[j]));
                            else
                                static_cast<float *>(p.y)[m * p.ldy + n] = __uint_as_float(r[j]);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&accempty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * ACC_COLS);
    }
}

}  // namespace qmmtc

bool qmm_tc_supported(const QmmArgs &a, const char **why) {
    auto no = [&](const char *r) { if (why) *why = r; return false; };
    if (a.bits != 4 && a.bits != 8) return no("qmm_tc: bits must be 4 or 8");
    if (a.group != 64) return no("qmm_tc: group_size must be 64");
    if (!a.x_bf16 || !a.p_bf16) return no("qmm_tc: activations and parameters must be bf16");
    if (a.M < 64) return no("qmm_tc: M < 64");
    if (a.K % 512) return no("qmm_tc: K must be a multiple of 512");
    if (a.x.col_stride != 1 || a.w.col_stride != 1 || a.s.col_stride != 1 || a.b.col_stride != 1)
        return no("qmm_tc: inputs need unit column stride");
    auto al = [](const void *p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    if (!al(a.x.ptr, 16) || (a.x.row_stride * 2) % 16) return no("qmm_tc: x rows must be 16-byte aligned");
    if (!al(a.w.ptr, 16) || (a.w.row_stride * 4) % 16) return no("qmm_tc: packed rows must be 16-byte aligned");
    if (!al(a.s.ptr, 16) || !al(a.b.ptr, 16) || (a.s.row_stride * 2) % 16 || (a.b.row_stride * 2) % 16)
        return no("qmm_tc: parameter rows must be 16-byte aligned");
    if (a.M >= (int64_t(1) << 31) || a.N >= (int64_t(1) << 31)) return no("qmm_tc: size beyond 32-bit indexing");
    return true;
}

template <int BITS>
static cudaError_t launch_bits(const QmmArgs &a, unsigned *status, cudaStream_t stream) {
    using C = qmmtc::Cfg<BITS>;
    qmmtc::Params p{};
    p.s = static_cast<const uint16_t *>(a.s.ptr);
    p.lds = a.s.row_stride;
    p.b = static_cast<const uint16_t *>(a.b.ptr);
    p.ldb = a.b.row_stride;
    p.y = a.y;
    p.ldy = a.ldy;
    p.status = status;
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(a.N);
    p.K = static_cast<int>(a.K);
    p.m_blocks = static_cast<int>((a.M + qmmtc::BX - 1) / qmmtc::BX);
    p.n_blocks = static_cast<int>((a.N + qmmtc::BW - 1) / qmmtc::BW);
    p.tiles = p.m_blocks * p.n_blocks;
    p.y_bf16 = a.y_bf16;
    const CUtensorMap *xm, *wm;
    if (!(xm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x.ptr, a.K, a.M, a.x.row_stride * 2, qmmtc::BK,
                                    qmmtc::BX, CU_TENSOR_MAP_SWIZZLE_128B)) ||
        !(wm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w.ptr, a.K * BITS / 32, a.N, a.w.row_stride * 4,
                                    qmmtc::BK * BITS / 32, qmmtc::BW, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return cudaErrorInvalidValue;
    auto kern = qmmtc::qmm_tc_kernel<BITS>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(kern), C::SMEM);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const int grid = std::min(p.tiles, sms);
    kern<<<grid, qmmtc::THREADS, C::SMEM, stream>>>(*xm, *wm, p);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_qmm_tc(const QmmArgs &a, void *workspace, cudaStream_t stream) {
    unsigned *status = static_cast<unsigned *>(workspace);
    return a.bits == 4 ? launch_bits<4>(a, status, stream) : launch_bits<8>(a, status, stream);
}

}  // namespace afb
