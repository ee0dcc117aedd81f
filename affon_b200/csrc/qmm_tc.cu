// Prefill qmm on tcgen05 tensor cores (placeholder until the kernel lands).
#include "internal.h"

namespace afb {

bool qmm_tc_supported(const QmmArgs &a, const char **why) {
    (void)a;
    if (why) *why = "qmm_tc: not available in this build";
    return false;
}

cudaError_t launch_qmm_tc(const QmmArgs &a, cudaStream_t stream) {
    (void)a;
    (void)stream;
    return cudaErrorNotSupported;
}

}  // namespace afb
