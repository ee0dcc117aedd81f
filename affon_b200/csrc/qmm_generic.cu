// Generic strided quantized matmul: every contract case the fast kernels do not
// take (2-bit, any group size, f32 activations or parameters, transposed /
// sliced / strided views).  This is the B200 counterpart of the reference's
// generic `cuda_quantized_matmul` candidate (docs/core/quantized-inference.md:
// 177-181: "reads logical strides and byte offsets directly and accumulates
// in f32").  One thread owns one output element and walks K in ascending
// order with the CPU kernel's operation order (decode s*q+b, then acc+x*w,
// every step rounded, no contraction), so its results are bit-identical to the
// scalar reference restated in oracle/qmm_ref.c.
#include "common.cuh"
#include "internal.h"

namespace afb {
namespace {

template <bool BF16>
__device__ __forceinline__ float load_elem(const View &v, int64_t r, int64_t c) {
    int64_t e = r * v.row_stride + c * v.col_stride;
    if (BF16) return bf16_bits_to_f32(static_cast<const uint16_t *>(v.ptr)[e]);
    return static_cast<const float *>(v.ptr)[e];
}

template <bool XB, bool PB>
__global__ void __launch_bounds__(256) qmm_generic_kernel(QmmArgs a) {
    int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= a.M * a.N) return;
    // Consecutive threads take consecutive n so weight rows are spread over the
    // warp and the activation row is shared.
    int64_t m = idx / a.N, n = idx % a.N;
    const int bits = a.bits;
    const int64_t per_word = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const uint32_t *w = static_cast<const uint32_t *>(a.w.ptr);
    float acc = 0.0f;
    for (int64_t k = 0; k < a.K; ++k) {
        int64_t g = k / a.group;
        uint32_t word = w[n * a.w.row_stride + (k / per_word) * a.w.col_stride];
        float q = static_cast<float>((word >> ((k % per_word) * bits)) & mask);
        float weight = __fadd_rn(__fmul_rn(load_elem<PB>(a.s, n, g), q), load_elem<PB>(a.b, n, g));
        acc = __fadd_rn(acc, __fmul_rn(load_elem<XB>(a.x, m, k), weight));
    }
    if (a.y_bf16)
        static_cast<uint16_t *>(a.y)[m * a.ldy + n] = f32_to_bf16_bits(acc);
    else
        static_cast<float *>(a.y)[m * a.ldy + n] = acc;
}

}  // namespace

cudaError_t launch_qmm_generic(const QmmArgs &a, cudaStream_t stream) {
    int64_t total = a.M * a.N;
    dim3 block(256);
    dim3 grid(static_cast<unsigned>((total + 255) / 256));
    if (a.x_bf16 && a.p_bf16) qmm_generic_kernel<true, true><<<grid, block, 0, stream>>>(a);
    else if (a.x_bf16) qmm_generic_kernel<true, false><<<grid, block, 0, stream>>>(a);
    else if (a.p_bf16) qmm_generic_kernel<false, true><<<grid, block, 0, stream>>>(a);
    else qmm_generic_kernel<false, false><<<grid, block, 0, stream>>>(a);
    count_launch();
    return cudaGetLastError();
}

}  // namespace afb
