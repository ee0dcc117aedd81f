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

// Decode qmv for M <= 16, bits in {4, 8}, group 64, bf16 x/s/b, dense rows.
struct QmvPlan {
    int splits;      // K splits (>= 1; 0 = not plannable): x slices that fit shared memory
    int ks;          // K per split
    int grid_n;      // persistent CTAs
    int stages;      // shared-memory ring depth
    int max_slots;   // partial-sum slots per block in the workspace
    int smem_bytes;
};

// Context workspace layout: [0, 256) device status words (a bounded wait that
// gives up writes there); [kCounterOffset, kPartialOffset) split-K arrival
// counters, zero between launches; [kPartialOffset, ...) f32 partial sums.
constexpr size_t kCounterOffset = 256;
constexpr int64_t kMaxTiles = 262144;
constexpr size_t kPartialOffset = kCounterOffset + size_t(kMaxTiles) * 4;
bool qmv_supported(const QmmArgs &a, const char **why);
QmvPlan qmv_plan(const QmmArgs &a, int num_sms, size_t workspace_bytes);
size_t qmv_workspace_bytes(const QmmArgs &a, const QmvPlan &p);
cudaError_t launch_qmv(const QmmArgs &a, const QmvPlan &p, void *workspace, cudaStream_t stream);

// Prefill qmm on tcgen05 tensor cores (M >= 64), bf16 x/s/b, 4/8-bit, group 64.
bool qmm_tc_supported(const QmmArgs &a, const char **why);
cudaError_t launch_qmm_tc(const QmmArgs &a, void *workspace, cudaStream_t stream);

void count_launch(uint64_t n = 1);

}  // namespace afb

struct affon_b200_qmm_desc;
namespace afb {
// Descriptor validation, argument resolution and the thread-local error
// message of the C ABI (abi.cu), for other entry points of the library.
int validate_qmm_desc(const affon_b200_qmm_desc *d);
QmmArgs qmm_args_from_desc(const affon_b200_qmm_desc *d, const void *x, const void *w, const void *s, const void *b,
                           void *y);
int set_error(int status, const char *msg);
int set_cuda_error(cudaError_t e, const char *what);
void clear_error();

}  // namespace afb
