// Kernels of the synthetic Llama-shaped decoder around the quantized
// linears: grouped-query decode attention with RoPE and KV-cache append fused
// in, the embedding gather that starts a step, and the argmax finalisation
// that ends it.  The reference has no quantized decoder (its Llama program,
// packages/@affon/models/src/llama/model.ts:64-78, uses dense matmuls); these
// kernels make the BASELINE decoder configurations runnable around the
// quantized_matmul kernels.
//
// Decode attention, one CTA per (128-position chunk, KV head, batch row):
// TMA loads the chunk's K and V rows (two 64-column boxes each, 128-byte
// swizzle) while the CTA rotates its GQA group's queries.  The CTA holding the
// current position also rotates the new key, writes key and value into the
// cache (bf16) and uses them directly.  Scores and softmax are f32 on the CUDA
// cores; each CTA leaves (max, sum, unnormalised output) per head, and the
// last CTA of a (batch, KV head) -- per-pair arrival counter -- merges the
// chunks in chunk order, so the result does not depend on scheduling.
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace afb {
namespace dec {

constexpr int HD = 128;        // head dimension
constexpr int CH = 128;        // positions per chunk (CTA)
constexpr int THREADS = 128;
constexpr int BOX_BYTES = CH * 64 * 2;  // one 64-column half of a K or V chunk

struct AttnParams {
    const uint16_t *qkv;
    int64_t ld_qkv;
    int q_off, k_off, v_off;
    uint16_t *kc, *vc;             // this layer's cache: [B][KVH][cap][HD]
    const float *cos_t, *sin_t;    // [cap][HD/2]
    const int *pos;
    uint16_t *out;
    int64_t ld_out;
    float *partial;
    unsigned *counters;
    unsigned *status;
    int B, QH, KVH, cap, max_chunks;
    float scale;
    int out_pair_order;
};

template <int G>
__global__ void __launch_bounds__(THREADS) decode_attention_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                   const __grid_constant__ CUtensorMap vmap,
                                                                   AttnParams p) {
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char *ks = smem;                        // 2 boxes
    char *vs = ks + 2 * BOX_BYTES;          // 2 boxes
    float *qs = reinterpret_cast<float *>(vs + 2 * BOX_BYTES);  // [G][HD]
    float *ps = qs + G * HD;                // [G][CH]
    float *knew = ps + G * CH;              // [HD]
    float *vnew = knew + HD;                // [HD]
    float *stat = vnew + HD;                // m[G], l[G]
    uint64_t *bar = reinterpret_cast<uint64_t *>(stat + 2 * G + 2);
    volatile int *flag = reinterpret_cast<volatile int *>(bar + 1);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int pos = *p.pos;
    const int n_chunks = pos / CH + 1;
    if (c >= n_chunks) return;
    const int c0 = c * CH;
    const int len = min(CH, pos + 1 - c0);
    const int row0 = (b * p.KVH + kvh) * p.cap + c0;

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(bar, 4 * BOX_BYTES);
        tma_load_2d(ks, &kmap, bar, 0, row0);
        tma_load_2d(ks + BOX_BYTES, &kmap, bar, 64, row0);
        tma_load_2d(vs, &vmap, bar, 0, row0);
        tma_load_2d(vs + BOX_BYTES, &vmap, bar, 64, row0);
    }
    // Rotated, pre-scaled queries of the GQA group (rotate-half RoPE: pairs
    // (d, d+64) with angle pos * theta^(-2d/HD)).
    const uint16_t *qrow = p.qkv + b * p.ld_qkv + p.q_off + kvh * G * HD;
    const float *cs = p.cos_t + static_cast<int64_t>(pos) * (HD / 2), *sn = p.sin_t + static_cast<int64_t>(pos) * (HD / 2);
    for (int i = tid; i < G * (HD / 2); i += THREADS) {
        const int h = i / (HD / 2), d = i % (HD / 2);
        const float a = bf16_bits_to_f32(qrow[h * HD + d]), bb = bf16_bits_to_f32(qrow[h * HD + d + HD / 2]);
        qs[h * HD + d] = (a * cs[d] - bb * sn[d]) * p.scale;
        qs[h * HD + d + HD / 2] = (bb * cs[d] + a * sn[d]) * p.scale;
    }
    const bool has_new = (pos >= c0) && (pos < c0 + CH);
    if (has_new) {  // rotate the new key, write key and value rows into the cache
        const uint16_t *krow = p.qkv + b * p.ld_qkv + p.k_off + kvh * HD;
        const uint16_t *vrow = p.qkv + b * p.ld_qkv + p.v_off + kvh * HD;
        const int64_t crow = static_cast<int64_t>((b * p.KVH + kvh) * p.cap + pos) * HD;
        if (tid < HD / 2) {
            const int d = tid;
            const float a = bf16_bits_to_f32(krow[d]), bb = bf16_bits_to_f32(krow[d + HD / 2]);
            const uint16_t r0 = f32_to_bf16_bits(a * cs[d] - bb * sn[d]);
            const uint16_t r1 = f32_to_bf16_bits(bb * cs[d] + a * sn[d]);
            p.kc[crow + d] = r0;
            p.kc[crow + d + HD / 2] = r1;
            knew[d] = bf16_bits_to_f32(r0);
            knew[d + HD / 2] = bf16_bits_to_f32(r1);
        }
        const uint16_t v = vrow[tid];
        p.vc[crow + tid] = v;
        vnew[tid] = bf16_bits_to_f32(v);
    }
    __syncthreads();
    volatile int abort_flag = 0;
    mbar_wait(bar, 0, &abort_flag, p.status);

    // Scores: thread i <-> position c0 + i.  Row i of a box holds 64 columns in
    // 16-byte chunks stored at chunk ^ (i % 8).
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = -INFINITY;
    if (tid < len) {
#pragma unroll
        for (int h = 0; h < G; ++h) sc[h] = 0.0f;
        const bool fresh = (c0 + tid == pos);
        for (int j = 0; j < HD / 8; ++j) {
            float kv[8];
            if (fresh) {
#pragma unroll
                for (int e = 0; e < 8; ++e) kv[e] = knew[j * 8 + e];
            } else {
                const char *box = ks + (j >> 3) * BOX_BYTES;
                const uint4 u = *reinterpret_cast<const uint4 *>(box + tid * 128 + (((j & 7) ^ (tid & 7)) << 4));
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    kv[2 * e] = __uint_as_float(w[e] << 16);
                    kv[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
                }
            }
#pragma unroll
            for (int h = 0; h < G; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e) sc[h] = fmaf(qs[h * HD + j * 8 + e], kv[e], sc[h]);
        }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) ps[h * CH + tid] = sc[h];
    __syncthreads();
    // Softmax statistics: warp w handles heads w, w+4, ...
    for (int hh = warp; hh < G; hh += THREADS / 32) {
        float v[CH / 32], mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < CH / 32; ++k) { v[k] = ps[hh * CH + lane + 32 * k]; mx = fmaxf(mx, v[k]); }
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < CH / 32; ++k) {
            const float e = (v[k] == -INFINITY) ? 0.0f : __expf(v[k] - mx);
            ps[hh * CH + lane + 32 * k] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) { stat[hh] = mx; stat[G + hh] = sum; }
    }
    __syncthreads();
    // Unnormalised outputs: thread d accumulates o[h][d] over the chunk.
    float o[G];
#pragma unroll
    for (int h = 0; h < G; ++h) o[h] = 0.0f;
    {
        const int d = tid, box = d >> 6, col = d & 63, chunk = col >> 3, within = (col & 7) * 2;
        const char *vb = vs + box * BOX_BYTES;
        for (int i = 0; i < len; ++i) {
            float vv;
            if (c0 + i == pos)
                vv = vnew[d];
            else
                vv = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(vb + i * 128 + ((chunk ^ (i & 7)) << 4) + within));
#pragma unroll
            for (int h = 0; h < G; ++h) o[h] = fmaf(ps[h * CH + i], vv, o[h]);
        }
    }
    // Partial record of this chunk: m[G], l[G], o[G][HD].
    const int pair = b * p.KVH + kvh;
    float *rec = p.partial + (static_cast<int64_t>(pair) * p.max_chunks + c) * (G * (HD + 2));
    if (tid < G) { rec[tid] = stat[tid]; rec[G + tid] = stat[G + tid]; }
#pragma unroll
    for (int h = 0; h < G; ++h) rec[2 * G + h * HD + tid] = o[h];
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    __syncthreads();
    if (tid == 0) *flag = (atomicAdd(&p.counters[pair], 1u) == static_cast<unsigned>(n_chunks - 1)) ? 1 : 0;
    __syncthreads();
    if (!*flag) return;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    // Merge the chunks in order.  Output column of this thread: d, or its
    // slot in the 4-bit qmv pair order (within 8 columns: 0 4 1 5 2 6 3 7).
    const int e8 = tid & 7;
    const int out_col = p.out_pair_order ? (tid & ~7) + (e8 < 4 ? 2 * e8 : 2 * (e8 - 4) + 1) : tid;
    const float *recs = p.partial + static_cast<int64_t>(pair) * p.max_chunks * (G * (HD + 2));
#pragma unroll
    for (int h = 0; h < G; ++h) {
        float M = -INFINITY;
        for (int cc = 0; cc < n_chunks; ++cc) M = fmaxf(M, __ldcg(&recs[cc * (G * (HD + 2)) + h]));
        float L = 0.0f, O = 0.0f;
        for (int cc = 0; cc < n_chunks; ++cc) {
            const float *r = recs + cc * (G * (HD + 2));
            const float w = __expf(__ldcg(&r[h]) - M);
            L = fmaf(__ldcg(&r[G + h]), w, L);
            O = fmaf(__ldcg(&r[2 * G + h * HD + tid]), w, O);
        }
        p.out[b * p.ld_out + (kvh * G + h) * HD + out_col] = f32_to_bf16_bits(O / L);
    }
    if (tid == 0) atomicExch(&p.counters[pair], 0u);
}

// h[b][:] = table[tokens[b]][:] (bf16 -> f32), the per-16-column sums of
// squares of h for the first norm, and a cleared argmax buffer.
__global__ void embed_kernel(const uint16_t *table, int64_t ld_table, const int *tokens, int B, int D, float *h,
                             float *ss_out, unsigned long long *amax) {
    const int b = blockIdx.y;
    const int tile = blockIdx.x * (blockDim.x / 16) + threadIdx.x / 16;  // 16 columns per tile
    const int col = tile * 16 + (threadIdx.x & 15);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x < B) amax[threadIdx.x] = 0ull;
    float v = 0.0f;
    if (col < D) {
        v = bf16_bits_to_f32(table[static_cast<int64_t>(tokens[b]) * ld_table + col]);
        h[static_cast<int64_t>(b) * D + col] = v;
    }
    float sq = v * v;
#pragma unroll
    for (int o = 8; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 15) == 0 && col < D) ss_out[tile * 16 + b] = sq;
}

// tokens[b] = argmax index from the packed maxima; history[step][b] keeps it;
// the position advances by one.
__global__ void finalize_kernel(const unsigned long long *amax, int B, int *tokens, int *history, int *pos,
                                int *step) {
    const int b = threadIdx.x;
    const int s = *step;
    if (b < B) {
        const int tok = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(amax[b] & 0xFFFFFFFFull));
        tokens[b] = tok;
        if (history) history[s * B + b] = tok;
    }
    __syncthreads();
    if (b == 0) {
        *pos += 1;
        *step = s + 1;
    }
}

}  // namespace dec

cudaError_t launch_decode_attention(const DecodeAttnArgs &a, void *workspace, cudaStream_t stream) {
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
    p.max_chunks = (a.capacity + dec::CH - 1) / dec::CH;
    p.scale = a.scale;
    p.out_pair_order = a.out_pair_order;
    char *ws = static_cast<char *>(workspace);
    p.status = reinterpret_cast<unsigned *>(ws);
    p.counters = reinterpret_cast<unsigned *>(ws + kCounterOffset);
    p.partial = reinterpret_cast<float *>(ws + kPartialOffset);
    const uint64_t rows = static_cast<uint64_t>(a.batch) * a.kv_heads * a.capacity;
    const CUtensorMap *km = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k_cache, dec::HD, rows,
                                                 dec::HD * 2, 64, dec::CH, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap *vm = cached_tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.v_cache, dec::HD, rows,
                                                 dec::HD * 2, 64, dec::CH, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!km || !vm) return cudaErrorInvalidValue;
    const int smem = 1024 + 4 * dec::BOX_BYTES + (G * dec::HD + G * dec::CH + 2 * dec::HD + 2 * G + 2) * 4 + 64;
    dim3 grid(p.max_chunks, a.kv_heads, a.batch);
    cudaError_t e;
    switch (G) {
    case 4:
        if ((e = ensure_smem_attr(reinterpret_cast<const void *>(dec::decode_attention_kernel<4>), smem)) != cudaSuccess)
            return e;
        dec::decode_attention_kernel<4><<<grid, dec::THREADS, smem, stream>>>(*km, *vm, p);
        break;
    case 8:
        if ((e = ensure_smem_attr(reinterpret_cast<const void *>(dec::decode_attention_kernel<8>), smem)) != cudaSuccess)
            return e;
        dec::decode_attention_kernel<8><<<grid, dec::THREADS, smem, stream>>>(*km, *vm, p);
        break;
    default:
        return cudaErrorInvalidValue;
    }
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_embed(const void *table, int64_t ld_table, const int *tokens, int B, int D, float *h, float *ss_out,
                         unsigned long long *amax, cudaStream_t stream) {
    const int threads = 256;  // 16 tiles of 16 columns per block
    dim3 grid((D + threads - 1) / threads, B);
    dec::embed_kernel<<<grid, threads, 0, stream>>>(static_cast<const uint16_t *>(table), ld_table, tokens, B, D, h,
                                                   ss_out, amax);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_finalize(const unsigned long long *amax, int B, int *tokens, int *history, int *pos, int *step,
                            cudaStream_t stream) {
    dec::finalize_kernel<<<1, 32 * ((B + 31) / 32), 0, stream>>>(amax, B, tokens, history, pos, step);
    count_launch();
    return cudaGetLastError();
}

}  // namespace afb
