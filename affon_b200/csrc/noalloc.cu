// Allocation-free entry point for the decode qmv.
//
// Some callers cannot let a library allocate device memory: a runtime that
// reserves every byte of the GPU in its own arena at start-up and forbids
// allocations behind its back, or a plugin host whose allocator is the only
// one allowed to call into the driver.  The regular entry points need an
// affon_b200 context, and creating one allocates the split-K workspace.
// affon_b200_qmv_noalloc() instead keeps the decode qmv's scratch (status
// word, per-block arrival counters and partial sums) in the static device
// array below, which every GPU that loads this library holds until the
// process exits.  affon_b200_qmv_noalloc_status() reads that array's status
// word back, so such a caller can still learn that a bounded wait gave up.
//
// The array's name in host code is only a host-side stand-in for the
// symbol, never a device address; the device address is looked up once per
// device with cudaGetSymbolAddress, with that device current, on the first
// call made on it, and cached.  That first call per device should therefore
// come before any stream capture.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/affon_b200.h"
#include "internal.h"

namespace {

// 8 MiB: the status word, 1 MiB of arrival counters and ~7 MiB of partial
// sums (kCounterOffset / kPartialOffset in internal.h lay it out).
constexpr size_t kScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_qmv_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of g_qmv_scratch on the current device (looked up once).
int scratch_address(int device, void **out) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[device]) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_qmv_scratch);
        if (e != cudaSuccess) return afb::set_cuda_error(e, "cudaGetSymbolAddress(qmv scratch)");
        g_scratch_addr[device] = ptr;
    }
    *out = g_scratch_addr[device];
    return AFFON_B200_OK;
}

}  // namespace

extern "C" int affon_b200_qmv_noalloc(const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                                      const void *s, const void *b, void *y, void *cuda_stream) {
    afb::clear_error();
    int rc = afb::validate_qmm_desc(desc);
    if (rc) return rc;
    if (!x || !w || !s || !b || !y) return afb::set_error(AFFON_B200_INVALID_ARG, "qmv_noalloc: null buffer");
    if (desc->numerical_policy == AFFON_B200_POLICY_EXACT_ONLY)
        return afb::set_error(AFFON_B200_POLICY_REJECTED,
                              "numericalPolicy exact_only rejects cuda_quantized_matmul (numerical class reassociated)");
    const afb::QmmArgs a = afb::qmm_args_from_desc(desc, x, w, s, b, y);
    const char *why = "";
    if (!afb::qmv_supported(a, &why)) return afb::set_error(AFFON_B200_UNSUPPORTED, why);
    int device = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return afb::set_cuda_error(e, "cudaGetDevice");
    if (device < 0 || device >= kMaxDevices) return afb::set_error(AFFON_B200_UNSUPPORTED, "qmv_noalloc: device ordinal");
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
        return afb::set_cuda_error(e, "cudaDeviceGetAttribute");
    const afb::QmvPlan plan = afb::qmv_plan(a, sms, kScratchBytes);
    if (plan.splits < 1)
        return afb::set_error(AFFON_B200_UNSUPPORTED,
                              "qmv_noalloc: M*N too large for the 8 MiB static scratch (its partial sums do not fit); "
                              "use affon_b200_qmm with a context");
    void *scratch = nullptr;
    if ((rc = scratch_address(device, &scratch))) return rc;
    cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
    // The array keeps the previous call's contents: clear the status word and
    // the arrival and completion counters this launch can touch before it runs.
    const size_t counters = (static_cast<size_t>(a.N) + 127) / 128 * sizeof(unsigned);
    if ((e = cudaMemsetAsync(scratch, 0, afb::kCounterOffset + counters, stream)) != cudaSuccess ||
        (e = cudaMemsetAsync(static_cast<char *>(scratch) + afb::kCounterOffset + afb::kMaxTiles / 2 * sizeof(unsigned),
                             0, counters, stream)) != cudaSuccess)
        return afb::set_cuda_error(e, "cudaMemsetAsync(qmv scratch)");
    if ((e = afb::launch_qmv(a, plan, scratch, stream)) != cudaSuccess) return afb::set_cuda_error(e, "qmv launch");
    return AFFON_B200_OK;
}

extern "C" int affon_b200_qmv_noalloc_status(void *cuda_stream, uint32_t *status_out) {
    afb::clear_error();
    if (!status_out) return afb::set_error(AFFON_B200_INVALID_ARG, "qmv_noalloc_status: null output");
    *status_out = 0;
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(cuda_stream));
    if (e != cudaSuccess)
        return afb::set_cuda_error(e, "stream synchronize");
    // The status word is the array's first 4 bytes (kCounterOffset layout).
    unsigned status = 0;
    if ((e = cudaMemcpyFromSymbol(&status, g_qmv_scratch, sizeof status, 0, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return afb::set_cuda_error(e, "cudaMemcpyFromSymbol(qmv scratch status)");
    *status_out = status;
    if (status != 0)
        return afb::set_error(AFFON_B200_TIMEOUT, "qmv_noalloc: a bounded wait gave up; the last result is invalid");
    return AFFON_B200_OK;
}
