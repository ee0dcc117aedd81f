// Kernels of the synthetic Llama-shaped decoder around the quantized
// linears: grouped-query decode attention with RoPE and KV-cache append fused
// in, the embedding gather that starts a step, and the argmax finalisation
// that ends it.  The reference has no quantized decoder (its Llama program,
// packages/@affon/models/src/llama/model.ts:64-78, uses dense matmuls); these
// kernels make the BASELINE decoder configurations runnable around the
// quantized_matmul kernels.
//
// Decode attention (flash-decoding).  Grid (splits, KV head, batch row): each
// CTA takes an equal share of the context's 64-position tiles and streams
// them through a 3-stage ring filled by TMA (K and V, two 64-column boxes
// each, 128-byte swizzle).  Four consumer warps each own 16 positions of every
// tile and run both products on tensor cores (mma.sync m16n8k16, bf16 in, f32
// accumulate): S = Q K^T with the GQA group's G <= 8 query heads as the rows
// of the A operand (pre-rotated, pre-scaled by log2(e)/sqrt(d), rounded to
// bf16) and K fragments read with ldmatrix; an online softmax per warp in f32
// (exp2); the probabilities, rounded to bf16, go from the S accumulators
// straight into the A operand of O += P V, with V fragments from
// ldmatrix.trans.  Q and P enter the tensor cores as bf16 hi + lo pairs (the
// lo halves in the A rows 8..15 the at most 8 heads leave free), so the
// products keep ~16 significant bits; the cache and q/k/v are bf16.  The warps' (max, sum, O) are merged in shared memory; when
// the context is split over several CTAs, each writes its record and the last
// CTA of the (batch, KV head) pair -- an arrival counter, nobody waits --
// merges the records in split order, so the result does not depend on
// scheduling.  The CTA holding the current position rotates the new key,
// writes key and value into the cache (bf16) and patches them into its staged
// tile, since the tile's TMA may have read the old row.
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace afb {
namespace dec {

constexpr int HD = 128;                    // head dimension
constexpr int TILE = 64;                   // positions per ring stage
constexpr int STAGES = 3;
constexpr int CWARPS = 4;                  // consumer warps, 16 positions of each tile each
constexpr int THREADS = 32 * (CWARPS + 1);  // + one producer warp
constexpr int BOX = TILE * 128;            // one 64-column half of a K or V tile: 8 KB
constexpr int STAGE_BYTES = 4 * BOX;       // K lo, K hi, V lo, V hi
constexpr int MAX_SPLITS = 16;
constexpr float LOG2E = 1.4426950408889634f;

struct AttnParams {
    const uint16_t *qkv;
    int64_t ld_qkv;
    int q_off, k_off, v_off;
    uint16_t *kc, *vc;             // this layer's cache: [B][KVH][cap][HD]
    const float *cos_t, *sin_t;    // [cap][HD/2]
    const int *pos;
    uint16_t *out;
    int64_t ld_out;
    float *partial;                // [pair][split][G * (HD + 2)]
    unsigned *counters;            // [pair]
    unsigned *status;
    int B, QH, KVH, cap, splits;
    float scale;
    int out_pair_order;
};

// Byte offset of (row r, column c) of a 64-row x 128-dim bf16 tile stored as
// two 64-column boxes with the 128-byte swizzle.
__device__ __forceinline__ int tile_off(int r, int c) {
    return (c >> 6) * BOX + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2;
}

__device__ __forceinline__ int out_column(int d, int pair_order) {
    const int e = d & 7;
    return pair_order ? (d & ~7) + (e < 4 ? 2 * e : 2 * (e - 4) + 1) : d;
}

template <int G>
__global__ void __launch_bounds__(THREADS, 2) decode_attention_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                   const __grid_constant__ CUtensorMap vmap,
                                                                   AttnParams p) {
    extern __shared__ char smem_raw[];
    char *ring = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + STAGES * STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    volatile int *flag = reinterpret_cast<volatile int *>(empty + STAGES);
    volatile int *abort = flag + 1;
    // After the tile loop the ring holds the warps' records: m, l [CWARPS][8], o [CWARPS][8][HD].
    float *red_m = reinterpret_cast<float *>(ring);
    float *red_l = red_m + CWARPS * 8;
    float *red_o = red_l + CWARPS * 8;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    pdl_launch_dependents();
    pdl_wait();  // q/k/v and the position come from the preceding kernels
    const int pos = *p.pos;
    if (pos < 0 || pos >= p.cap) {  // no store, no TMA: report and leave
        if (tid == 0 && split == 0 && kvh == 0 && b == 0) atomicExch(p.status, static_cast<unsigned>(DEV_BOUNDS));
        return;
    }
    const int T = pos / TILE + 1;  // tiles holding positions 0..pos
    const int t0 = split * T / p.splits, t1 = (split + 1) * T / p.splits;
    const int64_t row_base = static_cast<int64_t>(b * p.KVH + kvh) * p.cap;
    const int pair = b * p.KVH + kvh;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CWARPS);
        }
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == CWARPS) {  // ------------------------------------------ producer
        if (lane == 0 && t1 > t0) {
            tma_prefetch_desc(&kmap);
            tma_prefetch_desc(&vmap);
            const uint64_t stream_policy = l2_evict_first();
            int stage = 0;
            uint32_t phase = 0, issued = 0, par = 0;
            for (int i = t0; i < t1; ++i) {
                if (!mbar_wait(&empty[stage], phase ^ 1, abort, p.status) || *abort) break;  // never re-arm after an abort
                char *dst = ring + stage * STAGE_BYTES;
                mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                const int row = static_cast<int>(row_base) + i * TILE;
                tma_load_2d_hint(dst, &kmap, &full[stage], 0, row, stream_policy);
                tma_load_2d_hint(dst + BOX, &kmap, &full[stage], 64, row, stream_policy);
                tma_load_2d_hint(dst + 2 * BOX, &vmap, &full[stage], 0, row, stream_policy);
                tma_load_2d_hint(dst + 3 * BOX, &vmap, &full[stage], 64, row, stream_policy);
                issued |= 1u << stage;
                par = (par & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
            for (int s = 0; s < STAGES; ++s)
                if (issued & (1u << s)) mbar_wait_drain(&full[s], (par >> s) & 1u);
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    const int g = lane >> 2, t = lane & 3;
    // Q fragments.  A rows 0..7 hold the query heads (rows g < G) rounded to
    // bf16, rows 8..15 the rounding remainders of the same heads, so one
    // m16n8k16 gives both halves of each score (C rows g and g + 8) and the
    // scores carry ~16 significant bits of the rotated f32 query.  k-step ks
    // covers dims 16 ks .. 16 ks + 15: a0/a1 = dims 16ks+2t..+1 (hi/lo),
    // a2/a3 = dims 16ks+2t+8..+9.  RoPE pairs (d, d + 64).
    uint32_t qa[8][4];
    {
        const float qs = p.scale * LOG2E;
        const uint16_t *qrow = p.qkv + b * p.ld_qkv + p.q_off + (kvh * G + (g < G ? g : 0)) * HD;
        const float *cs = p.cos_t + static_cast<int64_t>(pos) * (HD / 2);
        const float *sn = p.sin_t + static_cast<int64_t>(pos) * (HD / 2);
        auto rot = [&](int d) {
            const int dd = d & 63;
            const float a = bf16_bits_to_f32(qrow[dd]), c = bf16_bits_to_f32(qrow[dd + 64]);
            return g < G ? (d < 64 ? a * cs[dd] - c * sn[dd] : c * cs[dd] + a * sn[dd]) * qs : 0.0f;
        };
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int d0 = 16 * ks + 2 * t;
            split_bf16x2(rot(d0), rot(d0 + 1), qa[ks][0], qa[ks][1]);
            split_bf16x2(rot(d0 + 8), rot(d0 + 9), qa[ks][2], qa[ks][3]);
        }
    }
    float m_run = -INFINITY, l_run = 0.0f;  // row g: running max (log2 units) and this thread's share of the sum
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;

    const int i_new = pos / TILE, r_new = pos % TILE;
    int stage = 0;
    uint32_t phase = 0;
    for (int i = t0; i < t1; ++i) {
        mbar_wait(&full[stage], phase, abort, p.status);
        char *tile = ring + stage * STAGE_BYTES;
        if (i == i_new && warp == r_new / 16) {
            // The current position: rotate the new key, store key and value
            // (bf16) into the cache and into the staged tile.
            const uint16_t *krow = p.qkv + b * p.ld_qkv + p.k_off + kvh * HD;
            const uint16_t *vrow = p.qkv + b * p.ld_qkv + p.v_off + kvh * HD;
            const float *cs = p.cos_t + static_cast<int64_t>(pos) * (HD / 2);
            const float *sn = p.sin_t + static_cast<int64_t>(pos) * (HD / 2);
            uint16_t *kdst = p.kc + (row_base + pos) * HD, *vdst = p.vc + (row_base + pos) * HD;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int d = 2 * lane + e;  // 0..63
                const float a = bf16_bits_to_f32(krow[d]), c = bf16_bits_to_f32(krow[d + 64]);
                const uint16_t r0 = f32_to_bf16_bits(a * cs[d] - c * sn[d]);
                const uint16_t r1 = f32_to_bf16_bits(c * cs[d] + a * sn[d]);
                kdst[d] = r0;
                kdst[d + 64] = r1;
                *reinterpret_cast<uint16_t *>(tile + tile_off(r_new, d)) = r0;
                *reinterpret_cast<uint16_t *>(tile + tile_off(r_new, d + 64)) = r1;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int d = 4 * lane + e;
                const uint16_t v = vrow[d];
                vdst[d] = v;
                *reinterpret_cast<uint16_t *>(tile + 2 * BOX + tile_off(r_new, d)) = v;
            }
            __syncwarp();
        }
        // S = Q K^T for this warp's 16 positions (n-tiles of 8).
        const uint32_t kbase = smem_u32(tile), vbase = smem_u32(tile + 2 * BOX);
        float sc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
            const int r = warp * 16 + j * 8 + (lane & 7);
#pragma unroll
            for (int kp = 0; kp < 4; ++kp) {  // k-steps 2kp, 2kp+1 = dims 32kp .. 32kp+31
                const int c = 32 * kp + 8 * (lane >> 3);  // first dim of this lane's 8x8 matrix
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kbase + (c >> 6) * BOX + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4), b0, b1, b2, b3);
                mma_bf16_16816(sc[j], qa[2 * kp], b0, b1, sc[j]);
                mma_bf16_16816(sc[j], qa[2 * kp + 1], b2, b3, sc[j]);
            }
        }
        // Online softmax of row g over the 4 scores this thread holds.
        const int p0 = i * TILE + warp * 16 + 2 * t;
        float v[4] = {sc[0][0] + sc[0][2], sc[0][1] + sc[0][3], sc[1][0] + sc[1][2], sc[1][1] + sc[1][3]};
        const int pp[4] = {p0, p0 + 1, p0 + 8, p0 + 9};
        float mx = -INFINITY;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (pp[e] > pos) v[e] = -INFINITY;
            mx = fmaxf(mx, v[e]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float corr = m_new == -INFINITY ? 1.0f : exp2f(m_run - m_new);
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[e] = v[e] == -INFINITY ? 0.0f : exp2f(v[e] - m_new);
        l_run = l_run * corr + (pr[0] + pr[1]) + (pr[2] + pr[3]);
        m_run = m_new;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            o[n][0] *= corr;
            o[n][1] *= corr;
            o[n][2] *= corr;
            o[n][3] *= corr;
        }
        // O += P V: P is the A operand, hi in rows g (positions 2t..2t+1 and
        // 2t+8..+9) and the remainders in rows g + 8, like Q; the two halves
        // of O are added at the end.
        uint32_t pa[4];
        split_bf16x2(pr[0], pr[1], pa[0], pa[1]);
        split_bf16x2(pr[2], pr[3], pa[2], pa[3]);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {  // dims 16jj .. 16jj+15 = n-tiles 2jj, 2jj+1
            const int mtx = lane >> 3;
            const int r = warp * 16 + (mtx & 1) * 8 + (lane & 7);
            const int c = 16 * jj + 8 * (mtx >> 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_trans(vbase + (c >> 6) * BOX + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4), b0, b1, b2, b3);
            mma_bf16_16816(o[2 * jj], pa, b0, b1, o[2 * jj]);
            mma_bf16_16816(o[2 * jj + 1], pa, b2, b3, o[2 * jj + 1]);
        }
        fence_proxy_async_smem();  // ldmatrix reads before the stage's next TMA fill
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
    }
    // The warp's row sums, then its record for the CTA merge.
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    constexpr int CT = CWARPS * 32;
    named_bar_sync(1, CT);  // every warp is done with the ring
    if (g < G) {
        if (t == 0) {
            red_m[warp * 8 + g] = m_run;
            red_l[warp * 8 + g] = l_run;
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            red_o[(warp * 8 + g) * HD + 8 * n + 2 * t] = o[n][0] + o[n][2];
            red_o[(warp * 8 + g) * HD + 8 * n + 2 * t + 1] = o[n][1] + o[n][3];
        }
    }
    named_bar_sync(1, CT);
    // CTA result for (head h, dim d): threads take d = tid, all G heads.
    const int d = tid;
    float cm[G], cl[G], co[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) M = fmaxf(M, red_m[w * 8 + h]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) {
            const float wt = M == -INFINITY ? 0.0f : exp2f(red_m[w * 8 + h] - M);
            L = fmaf(red_l[w * 8 + h], wt, L);
            O = fmaf(red_o[(w * 8 + h) * HD + d], wt, O);
        }
        cm[h] = M;
        cl[h] = L;
        co[h] = O;
    }
    const int col = out_column(d, p.out_pair_order);
    if (p.splits == 1) {
#pragma unroll
        for (int h = 0; h < G; ++h) p.out[b * p.ld_out + (kvh * G + h) * HD + col] = f32_to_bf16_bits(co[h] / cl[h]);
        return;
    }
    constexpr int REC = G * (HD + 2);
    float *rec = p.partial + (static_cast<int64_t>(pair) * p.splits + split) * REC;
#pragma unroll
    for (int h = 0; h < G; ++h) {
        rec[2 * G + h * HD + d] = co[h];
        if (d == 0) {
            rec[h] = cm[h];
            rec[G + h] = cl[h];
        }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    named_bar_sync(1, CT);
    if (tid == 0) *flag = (atomicAdd(&p.counters[pair], 1u) == static_cast<unsigned>(p.splits - 1)) ? 1 : 0;
    named_bar_sync(1, CT);
    if (!*flag) return;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    // Last CTA of the pair: merge the splits in order (loads issued together).
    const float *recs = p.partial + static_cast<int64_t>(pair) * p.splits * REC;
#pragma unroll
    for (int h = 0; h < G; ++h) {
        float ms[MAX_SPLITS];
#pragma unroll
        for (int s2 = 0; s2 < MAX_SPLITS; ++s2) ms[s2] = s2 < p.splits ? __ldcg(recs + s2 * REC + h) : -INFINITY;
        float M = -INFINITY;
#pragma unroll
        for (int s2 = 0; s2 < MAX_SPLITS; ++s2) M = fmaxf(M, ms[s2]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int s2 = 0; s2 < MAX_SPLITS; ++s2) {
            if (s2 < p.splits) {
                const float wt = ms[s2] == -INFINITY ? 0.0f : exp2f(ms[s2] - M);
                L = fmaf(__ldcg(recs + s2 * REC + G + h), wt, L);
                O = fmaf(__ldcg(recs + s2 * REC + 2 * G + h * HD + d), wt, O);
            }
        }
        p.out[b * p.ld_out + (kvh * G + h) * HD + col] = f32_to_bf16_bits(O / L);
    }
    if (tid == 0) atomicExch(&p.counters[pair], 0u);
}

// h[b][:] = table[tokens[b]][:] (bf16 -> f32), the per-16-column sums of
// squares of h for the first norm ([D/16][kSsWidth]), and a cleared argmax
// buffer.  A token outside [0, vocab) reads row 0 instead and sets the status
// word.
__global__ void embed_kernel(const uint16_t *table, int64_t ld_table, int64_t vocab, const int *tokens, int B, int D,
                             float *h, float *ss_out, unsigned long long *amax, const uint16_t *gamma, uint16_t *x,
                             int64_t ld_x, int pair_order, unsigned *status) {
    pdl_wait();
    const int b = blockIdx.y;
    const int tile = blockIdx.x * (blockDim.x / 16) + threadIdx.x / 16;  // 16 columns per tile
    const int col = tile * 16 + (threadIdx.x & 15);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x < B) amax[threadIdx.x] = 0ull;
    int tok = tokens[b];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(status, static_cast<unsigned>(DEV_BOUNDS));
        tok = 0;
    }
    float v = 0.0f;
    if (col < D) {
        v = bf16_bits_to_f32(table[static_cast<int64_t>(tok) * ld_table + col]);
        h[static_cast<int64_t>(b) * D + col] = v;
        if (gamma) x[b * ld_x + out_column(col, pair_order)] = f32_to_bf16_bits(v * bf16_bits_to_f32(gamma[col]));
    }
    float sq = v * v;
#pragma unroll
    for (int o = 8; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 15) == 0 && col < D) ss_out[tile * kSsWidth + b] = sq;
}

// tokens[b] = argmax index from the packed maxima; history[step % rows][b]
// keeps it (a ring of the last `rows` steps); the position advances by one.
__global__ void finalize_kernel(const unsigned long long *amax, int B, int *tokens, int *history, int history_rows,
                                int *pos, int *step) {
    pdl_wait();
    const int b = threadIdx.x;
    const int s = *step;
    if (b < B) {
        const int tok = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(amax[b] & 0xFFFFFFFFull));
        tokens[b] = tok;
        if (history && history_rows > 0) history[(s % history_rows) * B + b] = tok;
    }
    __syncthreads();
    if (b == 0) {
        *pos += 1;
        *step = s + 1;
    }
}

}  // namespace dec

int attention_splits(int batch, int kv_heads, int capacity, int num_sms) {
    // All CTAs resident at once (two per SM) in a single wave, each with at
    // least two tiles of the longest context.
    const int pairs = batch * kv_heads;
    int s = 2 * num_sms / pairs;
    const int tiles = (capacity + dec::TILE - 1) / dec::TILE;
    s = s < tiles / 2 ? s : tiles / 2;
    s = s < dec::MAX_SPLITS ? s : dec::MAX_SPLITS;
    return s < 1 ? 1 : s;
}

size_t attention_workspace_bytes(int batch, int kv_heads, int q_heads, int capacity, int num_sms) {
    const int G = q_heads / kv_heads;
    return kPartialOffset + size_t(batch) * kv_heads * attention_splits(batch, kv_heads, capacity, num_sms) * G *
                                (dec::HD + 2) * 4;
}

cudaError_t launch_decode_attention(const DecodeAttnArgs &a, void *workspace, int num_sms, cudaStream_t stream,
                                    bool pdl) {
    if (a.head_dim != dec::HD || a.q_heads % a.kv_heads) return cudaErrorInvalidValue;
    const int G = a.q_heads / a.kv_heads;
    dec::AttnParams p{};
    p.qkv = static_cast<const uint16_t *>(a.qkv);
    p.ld_qkv = a.ld_qkv;
    p.q_off = a.q_off;
    p.k_off = a.k_off;
    p.v_off = a.v_off;
    p.kc = static_cast<uint16_t *>(a.k_cache);
    p.vc = static_cast<uint16_t *>(a.v_cache);
    p.cos_t = a.rope_cos;
    p.sin_t = a.rope_sin;
    p.pos = a.pos;
    p.out = static_cast<uint16_t *>(a.out);
    p.ld_out = a.ld_out;
    p.B = a.batch;
    p.QH = a.q_heads;
    p.KVH = a.kv_heads;
    p.cap = a.capacity;
    p.splits = attention_splits(a.batch, a.kv_heads, a.capacity, num_sms);
    p.scale = a.scale;
    p.out_pair_order = a.out_pair_order;
    char *ws = static_cast<char *>(workspace);
    p.status = reinterpret_cast<unsigned *>(ws);
    p.counters = reinterpret_cast<unsigned *>(ws + kCounterOffset);
    p.partial = reinterpret_cast<float *>(ws + kPartialOffset);
    const uint64_t rows = static_cast<uint64_t>(a.batch) * a.kv_heads * a.capacity;
    const CUtensorMap *km = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k_cache, dec::HD, rows,
                                                 dec::HD * 2, 64, dec::TILE, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap *vm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.v_cache, dec::HD, rows,
                                                 dec::HD * 2, 64, dec::TILE, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!km || !vm) return cudaErrorInvalidValue;
    const int smem = 1024 + dec::STAGES * dec::STAGE_BYTES + 2 * dec::STAGES * 8 + 16;
    dim3 grid(p.splits, a.kv_heads, a.batch);
    cudaError_t e;
    switch (G) {
    case 4:
        if ((e = ensure_smem_attr(reinterpret_cast<const void *>(dec::decode_attention_kernel<4>), smem)) != cudaSuccess)
            return e;
        e = launch_ex(dec::decode_attention_kernel<4>, grid, dim3(dec::THREADS), smem, stream, false, pdl, *km, *vm, p);
        break;
    case 8:
        if ((e = ensure_smem_attr(reinterpret_cast<const void *>(dec::decode_attention_kernel<8>), smem)) != cudaSuccess)
            return e;
        e = launch_ex(dec::decode_attention_kernel<8>, grid, dim3(dec::THREADS), smem, stream, false, pdl, *km, *vm, p);
        break;
    default:
        return cudaErrorInvalidValue;
    }
    count_launch();
    return e;
}

cudaError_t launch_embed(const void *table, int64_t ld_table, int64_t vocab, const int *tokens, int B, int D,
                         float *h, float *ss_out, unsigned long long *amax, const uint16_t *gamma, uint16_t *x,
                         int64_t ld_x, int pair_order, void *workspace, cudaStream_t stream, bool pdl) {
    const int threads = 256;  // 16 tiles of 16 columns per block
    dim3 grid((D + threads - 1) / threads, B);
    cudaError_t e = launch_ex(dec::embed_kernel, grid, dim3(threads), 0, stream, false, pdl,
                              static_cast<const uint16_t *>(table), ld_table, vocab, tokens, B, D, h, ss_out, amax,
                              gamma, x, ld_x, pair_order, static_cast<unsigned *>(workspace));
    count_launch();
    return e;
}

cudaError_t launch_finalize(const unsigned long long *amax, int B, int *tokens, int *history, int history_rows,
                            int *pos, int *step, cudaStream_t stream, bool pdl) {
    cudaError_t e = launch_ex(dec::finalize_kernel, dim3(1), dim3(32 * ((B + 31) / 32)), 0, stream, false, pdl, amax,
                              B, tokens, history, history_rows, pos, step);
    count_launch();
    return e;
}

}  // namespace afb
