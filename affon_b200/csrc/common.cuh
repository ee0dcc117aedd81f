// Shared device helpers for the sm_100a quantized-matmul kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define AFB_DEVICE __device__ __forceinline__

namespace afb {

AFB_DEVICE float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

// Round-to-nearest-even f32 -> bf16 bits (cvt.rn.bf16.f32).
AFB_DEVICE uint16_t f32_to_bf16_bits(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t *>(&h);
}

// Two f32 -> packed bf16x2 (low half = lo), one cvt.rn.bf16x2.f32.
AFB_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// (x0, x1) as bf16 pairs hi = bf16(x) and lo = bf16(x - hi): hi + lo carries
// ~16 significant bits of x.
AFB_DEVICE void split_bf16x2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    hi = pack_bf16x2(x0, x1);
    lo = pack_bf16x2(x0 - __uint_as_float(hi << 16), x1 - __uint_as_float(hi & 0xFFFF0000u));
}

// d = (a & b) | c
AFB_DEVICE uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Packed bf16x2 subtraction a - b (exact when the result is representable).
AFB_DEVICE uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

AFB_DEVICE uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Natural-order exact bf16 code pairs of a 4-bit word: (q0,q1), (q2,q3),
// (q4,q5), (q6,q7).  Even nibbles are gathered into the low half-word and odd
// ones into the high half-word (two delta swaps); each pair is then the bf16
// pair (128+q, 128+q') built by one logic op, minus 128 (exact).
AFB_DEVICE void dec4_nat(uint32_t w, uint32_t (&out)[4]) {
    uint32_t t = (w ^ (w >> 4)) & 0x00F000F0u;
    w ^= t ^ (t << 4);
    t = (w ^ (w >> 8)) & 0x0000FF00u;
    w ^= t ^ (t << 8);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        out[i] = bf16x2_sub(lop3_and_or(w >> (4 * i), 0x000F000Fu, 0x43004300u), 0x43004300u);
}
// Bytes i and i+1 of an 8-bit word as an exact bf16 pair (q, q'), through
// the f32 2^23 + q trick.
AFB_DEVICE uint32_t dec8_pair(uint32_t w, int i) {
    float f0 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i)) - 8388608.0f;
    float f1 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540u + i + 1)) - 8388608.0f;
    return pack_bf16x2(f0, f1);
}

// Streaming loads of packed weights: read-only path, no L1 allocation.
AFB_DEVICE uint2 ldg_stream_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
AFB_DEVICE uint4 ldg_stream_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
AFB_DEVICE uint2 ldg_nc_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
AFB_DEVICE uint4 ldg_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, f32 accumulate.
AFB_DEVICE void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// Four 8x8 b16 matrices from shared memory; lane l gives the address of row
// l % 8 of matrix l / 8, and receives elements (l / 4, 2 (l % 4) .. +1) of each
// matrix (the .trans form: the transposed matrices).
AFB_DEVICE void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
AFB_DEVICE void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

}  // namespace afb
