// C ABI of the affon_b200 library: contexts, validation, physical selection
// and dispatch for quantized_matmul.  See include/affon_b200.h.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/affon_b200.h"
#include "internal.h"
#include "sm100.cuh"


namespace afb {

static std::atomic<uint64_t> g_launches{0};
void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

}  // namespace afb

namespace {

thread_local std::string t_error;

int fail(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(AFFON_B200_CUDA_ERROR, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr size_t kDefaultWorkspace = size_t(64) << 20;

// Makes ctx->device current for the scope of one call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int env_device() {
    const char *v = getenv("AFFON_CUDA_DEVICE");
    if (!v || !*v) return 0;
    char *end = nullptr;
    long d = strtol(v, &end, 10);
    if (*end || d < 0) return -1;
    return static_cast<int>(d);
}

bool is_float_dtype(int d) { return d == AFFON_B200_F32 || d == AFFON_B200_BF16; }
size_t dtype_size(int d) { return d == AFFON_B200_BF16 ? 2 : 4; }

bool view_dense(const affon_b200_view &v) {
    return v.byte_offset == 0 && v.col_stride == 1 && v.row_stride == v.cols;
}

// Largest element index a view touches, plus one (strides are non-negative).
int64_t view_extent(const affon_b200_view &v) {
    return (v.rows - 1) * v.row_stride + (v.cols - 1) * v.col_stride + 1;
}

int validate_desc(const affon_b200_qmm_desc *d) {
    if (!d) return fail(AFFON_B200_INVALID_ARG, "quantized_matmul: null descriptor");
    if (d->struct_size != sizeof(affon_b200_qmm_desc))
        return fail(AFFON_B200_INVALID_ARG, "quantized_matmul: descriptor struct_size %u, expected %zu", d->struct_size,
                    sizeof(affon_b200_qmm_desc));
    // program.ts:483-484
    if (d->bits != 2 && d->bits != 4 && d->bits != 8)
        return fail(AFFON_B200_INVALID_SHAPE, "quantized_matmul bits must be 2, 4, or 8");
    if (d->group_size <= 0) return fail(AFFON_B200_INVALID_SHAPE, "quantized_matmul group_size must be a positive integer");
    // program.ts:486-487
    if (!is_float_dtype(d->x_dtype) || !is_float_dtype(d->param_dtype))
        return fail(AFFON_B200_INVALID_DTYPE,
                    "quantized_matmul requires f32/bf16 input, u32 weights, and matching f32/bf16 scales and biases");
    if (!is_float_dtype(d->y_dtype)) return fail(AFFON_B200_INVALID_DTYPE, "quantized_matmul result dtype must be f32 or bf16");
    const affon_b200_view *vs[5] = {&d->x, &d->w, &d->s, &d->b, &d->y};
    for (const affon_b200_view *v : vs) {
        if (v->rows < 0 || v->cols < 0 || v->row_stride < 0 || v->col_stride < 0 || v->byte_offset < 0)
            return fail(AFFON_B200_INVALID_ARG, "quantized_matmul: negative view extent, stride or offset");
    }
    // program.ts:488-492
    const int64_t rows = d->x.rows, inner = d->x.cols, outputs = d->w.rows;
    const int64_t per_word = 32 / d->bits;
    if (!rows || !inner || !outputs || inner % per_word || inner % d->group_size || d->w.cols != inner / per_word ||
        d->s.rows != outputs || d->s.cols != inner / d->group_size || d->b.rows != outputs ||
        d->b.cols != inner / d->group_size)
        return fail(AFFON_B200_INVALID_SHAPE, "quantized_matmul packed or group dimensions do not match input features");
    // Result spec f32 [rows, outputs] (program.ts:494).
    if (d->y.rows != rows || d->y.cols != outputs)
        return fail(AFFON_B200_INVALID_SHAPE, "quantized_matmul result view must be [%lld, %lld]", (long long)rows,
                    (long long)outputs);
    if (d->y.col_stride != 1 || d->y.row_stride < outputs)
        return fail(AFFON_B200_UNSUPPORTED, "quantized_matmul result view must have dense rows");
    if (rows > (int64_t(1) << 40) / inner || outputs > (int64_t(1) << 40) / inner || rows > (int64_t(1) << 40) / outputs)
        return fail(AFFON_B200_INVALID_SHAPE, "quantized_matmul dimensions overflow");
    if (d->dense_inputs) {
        // optimization-and-profiling.md:143-151: incompatible views fail with GuardMismatch.
        if (!view_dense(d->x) || !view_dense(d->w) || !view_dense(d->s) || !view_dense(d->b))
            return fail(AFFON_B200_GUARD_MISMATCH, "GuardMismatch: denseInputs requires dense, zero-offset inputs");
    }
    if (d->numerical_policy < 0 || d->numerical_policy > 2)
        return fail(AFFON_B200_INVALID_ARG, "quantized_matmul: unknown numerical policy %d", d->numerical_policy);
    return AFFON_B200_OK;
}

afb::QmmArgs make_args(const affon_b200_qmm_desc *d, const void *x, const void *w, const void *s, const void *b,
                       void *y) {
    afb::QmmArgs a{};
    auto view = [](const void *base, const affon_b200_view &v) {
        return afb::View{static_cast<const char *>(base) + v.byte_offset, v.row_stride, v.col_stride};
    };
    a.x = view(x, d->x);
    a.w = view(w, d->w);
    a.s = view(s, d->s);
    a.b = view(b, d->b);
    a.y = static_cast<char *>(y) + d->y.byte_offset;
    a.ldy = d->y.row_stride;
    a.M = d->x.rows;
    a.N = d->w.rows;
    a.K = d->x.cols;
    a.group = d->group_size;
    a.bits = d->bits;
    a.x_bf16 = d->x_dtype == AFFON_B200_BF16;
    a.p_bf16 = d->param_dtype == AFFON_B200_BF16;
    a.y_bf16 = d->y_dtype == AFFON_B200_BF16;
    return a;
}

enum Impl { IMPL_GENERIC = 0, IMPL_QMV = 1, IMPL_QMM_TC = 2, IMPL_QMM_EXACT = 3 };

struct Choice {
    Impl impl;
    afb::QmvPlan plan;
    int passes;  // qmv passes over 32-row slices of M
};

int select_impl(const affon_b200_qmm_desc *d, const afb::QmmArgs &a, int num_sms, size_t workspace,
                affon_b200_selection *sel, Choice *out) {
    // quantized-inference.md:175-177: quantized candidates are `reassociated`;
    // exact_only rejects them.
    if (d->numerical_policy == AFFON_B200_POLICY_EXACT_ONLY)
        return fail(AFFON_B200_POLICY_REJECTED,
                    "numericalPolicy exact_only rejects cuda_quantized_matmul (numerical class reassociated)");
    Choice c{IMPL_GENERIC, {}, 1};
    char reason[256];
    const char *why_qmv = "";
    afb::QmmArgs probe = a;
    probe.M = a.M < afb::kMaxQmvRows ? a.M : afb::kMaxQmvRows;
    const bool qmv_ok = afb::qmv_supported(probe, &why_qmv);
    const char *why_tc = "";
    const bool tc_ok = afb::qmm_tc_supported(a, &why_tc);
    const char *why_exact = "";
    bool exact_ok = afb::qmm_exact_supported(a, &why_exact);
    if (exact_ok && afb::qmm_exact_min_workspace(a) > workspace) {
        exact_ok = false;
        why_exact = "qmm_exact: the context workspace is too small";
    }
    afb::QmvPlan qplan{};
    if (qmv_ok) qplan = afb::qmv_plan(probe, num_sms, workspace);
    const bool qmv_plannable = qmv_ok && qplan.splits > 0;
    if (qmv_ok && !qmv_plannable) why_qmv = "qmv: no split fits shared memory and the context workspace";
    if (qmv_plannable && a.M <= afb::kMaxQmvRows) {
        c.impl = IMPL_QMV;
        c.plan = qplan;
        if (c.plan.variant >= 6)
            snprintf(reason, sizeof reason,
                     "M=%lld <= 32: decode qmv, %d-row whole-K blocks over %d CTAs, K split over the warps of a CTA, "
                     "%d-stage ring",
                     (long long)a.M, c.plan.rows, c.plan.grid_n, c.plan.stages);
        else
            snprintf(reason, sizeof reason,
                     "M=%lld <= 32: decode qmv, stream-K over %d CTAs, up to %d K segments per tile, %d-stage ring",
                     (long long)a.M, c.plan.grid_n, c.plan.max_slots, c.plan.stages);
    } else if (tc_ok && d->numerical_policy == AFFON_B200_POLICY_APPROXIMATE) {
        c.impl = IMPL_QMM_TC;
        snprintf(reason, sizeof reason, "M=%lld >= 64: tcgen05 qmm with bf16-rounded decoded weights", (long long)a.M);
    } else if (exact_ok) {
        c.impl = IMPL_QMM_EXACT;
        snprintf(reason, sizeof reason,
                 "M=%lld >= 64: tcgen05 qmm on exact codes, per-group f32 scales, bias term on tensor cores",
                 (long long)a.M);
    } else if (qmv_plannable && (a.M <= 64 || d->numerical_policy != AFFON_B200_POLICY_APPROXIMATE)) {
        c.impl = IMPL_QMV;
        c.passes = static_cast<int>((a.M + afb::kMaxQmvRows - 1) / afb::kMaxQmvRows);
        c.plan = qplan;
        snprintf(reason, sizeof reason, "M=%lld > 32: %d qmv passes over 32-row slices", (long long)a.M, c.passes);
    } else {
        snprintf(reason, sizeof reason, "generic strided kernel (%s; %s)", why_qmv, why_exact);
    }
    if (sel) {
        memset(sel, 0, sizeof *sel);
        if (c.impl == IMPL_QMV)
            snprintf(sel->implementation_id, sizeof sel->implementation_id, "cuda_quantized_matmul.sm100_qmv_b%d_g64",
                     d->bits);
        else if (c.impl == IMPL_QMM_TC)
            snprintf(sel->implementation_id, sizeof sel->implementation_id,
                     "cuda_quantized_matmul.sm100_qmm_tcgen05_b%d_g64", d->bits);
        else if (c.impl == IMPL_QMM_EXACT)
            snprintf(sel->implementation_id, sizeof sel->implementation_id,
                     "cuda_quantized_matmul.sm100_qmm_tcgen05_exact_b%d_g64", d->bits);
        else
            snprintf(sel->implementation_id, sizeof sel->implementation_id, "cuda_quantized_matmul.sm100_generic");
        sel->implementation_version = 1;
        sel->numerical_class = c.impl == IMPL_QMM_TC ? AFFON_B200_APPROXIMATE : AFFON_B200_REASSOCIATED;
        sel->splits = c.impl == IMPL_QMV ? c.plan.max_slots : 1;  // K segments combined per output tile
        snprintf(sel->reason, sizeof sel->reason, "%s", reason);
    }
    *out = c;
    return AFFON_B200_OK;
}

int launch(affon_b200_ctx *ctx, const afb::QmmArgs &a, const Choice &c) {
    cudaError_t e = cudaSuccess;
    switch (c.impl) {
    case IMPL_QMV: {
        for (int pass = 0; pass < c.passes && e == cudaSuccess; ++pass) {
            afb::QmmArgs slice = a;
            const int64_t m0 = int64_t(pass) * afb::kMaxQmvRows;
            slice.M = (a.M - m0) < afb::kMaxQmvRows ? (a.M - m0) : afb::kMaxQmvRows;
            slice.x.ptr = static_cast<const char *>(a.x.ptr) + m0 * a.x.row_stride * 2;
            slice.y = static_cast<char *>(a.y) + m0 * a.ldy * (a.y_bf16 ? 2 : 4);
            afb::QmvPlan plan = slice.M == afb::kMaxQmvRows || c.passes == 1
                                    ? c.plan
                                    : afb::qmv_plan(slice, ctx->num_sms, ctx->workspace_bytes);
            if (plan.splits < 1 || afb::qmv_workspace_bytes(slice, plan) > ctx->workspace_bytes)
                return fail(AFFON_B200_CUDA_ERROR, "qmv plan exceeds the context workspace");
            e = afb::launch_qmv(slice, plan, ctx->workspace, ctx->stream, nullptr, ctx->overlap);
        }
        break;
    }
    case IMPL_QMM_TC:
        e = afb::launch_qmm_tc(a, ctx->workspace, ctx->stream);
        break;
    case IMPL_QMM_EXACT:
        e = afb::launch_qmm_exact(a, ctx->workspace, ctx->workspace_bytes, ctx->stream);
        break;
    default:
        e = afb::launch_qmm_generic(a, ctx->stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul launch");
    return AFFON_B200_OK;
}

int grow(void **buf, size_t *have, size_t need) {
    if (*have >= need) return AFFON_B200_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *have = 0;
    size_t want = need < 256 ? 256 : need;
    cudaError_t e = cudaMalloc(buf, want);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    *have = want;
    return AFFON_B200_OK;
}

thread_local affon_b200_ctx *t_default_ctx = nullptr;

}  // namespace

// Shared with other translation units of the library (see internal.h).
namespace afb {
int validate_qmm_desc(const affon_b200_qmm_desc *d) { return validate_desc(d); }
QmmArgs qmm_args_from_desc(const affon_b200_qmm_desc *d, const void *x, const void *w, const void *s, const void *b,
                           void *y) {
    return make_args(d, x, w, s, b, y);
}
int set_error(int status, const char *msg) { return fail(status, "%s", msg); }
int set_cuda_error(cudaError_t e, const char *what) { return cuda_fail(e, what); }
void clear_error() { t_error.clear(); }
}  // namespace afb

extern "C" {

int affon_b200_abi_version(void) { return AFFON_B200_ABI_VERSION; }

const char *affon_b200_last_error(void) { return t_error.c_str(); }

uint64_t affon_b200_launch_count(void) { return afb::g_launches.load(); }

int affon_b200_ctx_create(int device_ordinal, void *cuda_stream, affon_b200_ctx **out) {
    if (!out) return fail(AFFON_B200_INVALID_ARG, "ctx_create: null output pointer");
    *out = nullptr;
    int dev = device_ordinal >= 0 ? device_ordinal : env_device();
    if (dev < 0) return fail(AFFON_B200_INVALID_ARG, "AFFON_CUDA_DEVICE must be a non-negative integer");
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) return fail(AFFON_B200_UNSUPPORTED, "backend unavailable: no CUDA device");
    if (dev >= count) return fail(AFFON_B200_INVALID_ARG, "CUDA device %d out of range (%d devices)", dev, count);
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, dev)) != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(AFFON_B200_UNSUPPORTED, "backend unavailable: affon_b200 requires sm_100 (found sm_%d%d)", prop.major,
                    prop.minor);
    DeviceGuard guard(dev);
    if (!guard.ok) return fail(AFFON_B200_CUDA_ERROR, "cudaSetDevice(%d) failed", dev);
    affon_b200_ctx *c = new affon_b200_ctx;
    c->device = dev;
    c->stream = static_cast<cudaStream_t>(cuda_stream);
    c->num_sms = prop.multiProcessorCount;
    int rc = affon_b200_ctx_reserve_workspace(c, kDefaultWorkspace);
    if (rc) {
        delete c;
        return rc;
    }
    *out = c;
    return AFFON_B200_OK;
}

int affon_b200_ctx_destroy(affon_b200_ctx *ctx) {
    if (!ctx) return AFFON_B200_OK;
    DeviceGuard guard(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    else cudaDeviceSynchronize();
    if (ctx->tp) afb::tp_release(ctx);
    if (ctx->workspace) cudaFree(ctx->workspace);
    for (void *p : ctx->stage)
        if (p) cudaFree(p);
    if (t_default_ctx == ctx) t_default_ctx = nullptr;
    delete ctx;
    return AFFON_B200_OK;
}

int affon_b200_ctx_set_stream(affon_b200_ctx *ctx, void *cuda_stream) {
    if (!ctx) return fail(AFFON_B200_INVALID_ARG, "null context");
    ctx->stream = static_cast<cudaStream_t>(cuda_stream);
    return AFFON_B200_OK;
}

int affon_b200_ctx_device(const affon_b200_ctx *ctx) { return ctx ? ctx->device : -1; }

int affon_b200_ctx_set_overlap(affon_b200_ctx *ctx, int enable) {
    if (!ctx) return fail(AFFON_B200_INVALID_ARG, "null context");
    ctx->overlap = enable != 0;
    return AFFON_B200_OK;
}

int affon_b200_debug_set_combine_wait(uint64_t limit_ns, uint32_t extra_arrivals) {
    afb::qmv_set_combine_wait(limit_ns, extra_arrivals);
    return AFFON_B200_OK;
}

int affon_b200_debug_set_slice_rows(int64_t rows) {
    if (rows < 0) return fail(AFFON_B200_INVALID_ARG, "slice rows must be >= 0");
    afb::qmm_exact_set_slice_cap(rows);
    return AFFON_B200_OK;
}

int affon_b200_ctx_reserve_workspace(affon_b200_ctx *ctx, size_t bytes) {
    if (!ctx) return fail(AFFON_B200_INVALID_ARG, "null context");
    if (bytes <= ctx->workspace_bytes) return AFFON_B200_OK;
    DeviceGuard guard(ctx->device);
    // The old workspace may still be in use by queued launches.
    if (ctx->workspace) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->workspace);
        ctx->workspace = nullptr;
        ctx->workspace_bytes = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->workspace, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "workspace cudaMalloc");
    // Split-K arrival counters must start at zero; launches leave them zero.
    if ((e = cudaMemset(ctx->workspace, 0, bytes)) != cudaSuccess) return cuda_fail(e, "workspace cudaMemset");
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(e, "workspace init");
    ctx->workspace_bytes = bytes;
    return AFFON_B200_OK;
}

int affon_b200_ctx_synchronize(affon_b200_ctx *ctx) {
    t_error.clear();
    if (!ctx) return fail(AFFON_B200_INVALID_ARG, "null context");
    DeviceGuard guard(ctx->device);
    cudaError_t e = ctx->stream ? cudaStreamSynchronize(ctx->stream) : cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
    unsigned status = 0;
    if ((e = cudaMemcpy(&status, ctx->workspace, sizeof status, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "status read");
    if (status != 0) {
        // A kernel that gave up may have left arrival counters behind: clear
        // the status word and the whole counter region for the next launch.
        if ((e = cudaMemset(ctx->workspace, 0, afb::kPartialOffset)) != cudaSuccess ||
            (e = cudaDeviceSynchronize()) != cudaSuccess)
            return cuda_fail(e, "status reset");
        if (status == afb::DEV_BOUNDS)
            return fail(AFFON_B200_INVALID_ARG,
                        "a kernel read a position or token outside its buffer and skipped it (device status %u)", status);
        return fail(AFFON_B200_TIMEOUT, "a kernel gave up a bounded wait (device status %u)", status);
    }
    return AFFON_B200_OK;
}

int affon_b200_validate(const affon_b200_qmm_desc *desc) {
    t_error.clear();
    return validate_desc(desc);
}

int affon_b200_select(const affon_b200_qmm_desc *desc, affon_b200_selection *out) {
    t_error.clear();
    int rc = validate_desc(desc);
    if (rc) return rc;
    // Selection needs only shapes, dtypes and alignment; use placeholder
    // 256-byte-aligned device addresses for the alignment rules.
    char *fake = reinterpret_cast<char *>(uintptr_t(1) << 40);
    afb::QmmArgs a = make_args(desc, fake, fake, fake, fake, fake);
    Choice c;
    return select_impl(desc, a, 148, kDefaultWorkspace, out, &c);
}

int affon_b200_qmm_explain(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                           const void *s, const void *b, void *y, affon_b200_selection *sel) {
    t_error.clear();
    if (!ctx) return fail(AFFON_B200_INVALID_ARG, "null context");
    int rc = validate_desc(desc);
    if (rc) return rc;
    if (!x || !w || !s || !b || !y) return fail(AFFON_B200_INVALID_ARG, "quantized_matmul: null buffer");
    afb::QmmArgs a = make_args(desc, x, w, s, b, y);
    Choice c;
    rc = select_impl(desc, a, ctx->num_sms, ctx->workspace_bytes, sel, &c);
    if (rc) return rc;
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(AFFON_B200_CUDA_ERROR, "cudaSetDevice(%d) failed", ctx->device);
    return launch(ctx, a, c);
}

int affon_b200_qmm(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                   const void *s, const void *b, void *y) {
    return affon_b200_qmm_explain(ctx, desc, x, w, s, b, y, nullptr);
}

int affon_b200_qmm_host(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                        const void *s, const void *b, void *y) {
    t_error.clear();
    if (!ctx) return fail(AFFON_B200_INVALID_ARG, "null context");
    int rc = validate_desc(desc);
    if (rc) return rc;
    if (!x || !w || !s || !b || !y) return fail(AFFON_B200_INVALID_ARG, "quantized_matmul: null buffer");
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(AFFON_B200_CUDA_ERROR, "cudaSetDevice(%d) failed", ctx->device);
    const void *host[4] = {x, w, s, b};
    const affon_b200_view *views[4] = {&desc->x, &desc->w, &desc->s, &desc->b};
    const size_t esz[4] = {dtype_size(desc->x_dtype), 4, dtype_size(desc->param_dtype), dtype_size(desc->param_dtype)};
    size_t bytes[5];
    for (int i = 0; i < 4; ++i) bytes[i] = views[i]->byte_offset + size_t(view_extent(*views[i])) * esz[i];
    const size_t ysz = dtype_size(desc->y_dtype);
    bytes[4] = desc->y.byte_offset + size_t(view_extent(desc->y)) * ysz;
    for (int i = 0; i < 5; ++i)
        if ((rc = grow(&ctx->stage[i], &ctx->stage_bytes[i], bytes[i]))) return rc;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 4 && e == cudaSuccess; ++i)
        e = cudaMemcpyAsync(ctx->stage[i], host[i], bytes[i], cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "host-to-device copy");
    afb::QmmArgs a = make_args(desc, ctx->stage[0], ctx->stage[1], ctx->stage[2], ctx->stage[3], ctx->stage[4]);
    Choice c;
    if ((rc = select_impl(desc, a, ctx->num_sms, ctx->workspace_bytes, nullptr, &c))) return rc;
    if ((rc = launch(ctx, a, c))) return rc;
    // Copy back only the rows of y (dense rows of N elements at row stride ldy).
    const size_t row_bytes = size_t(desc->y.cols) * ysz;
    e = cudaMemcpy2DAsync(static_cast<char *>(y) + desc->y.byte_offset, size_t(desc->y.row_stride) * ysz,
                          static_cast<char *>(ctx->stage[4]) + desc->y.byte_offset, size_t(desc->y.row_stride) * ysz,
                          row_bytes, size_t(desc->y.rows), cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "device-to-host copy");
    if ((e = cudaStreamSynchronize(ctx->stream)) != cudaSuccess) return cuda_fail(e, "stream synchronize");
    return AFFON_B200_OK;
}

int affon_b200_qmv_fused(affon_b200_ctx *ctx, const affon_b200_qmm_desc *desc, const void *x, const uint32_t *w,
                         const void *s, const void *b, void *y, const affon_b200_qmv_fusion *fusion) {
    t_error.clear();
    if (!ctx || !fusion || fusion->struct_size != sizeof(affon_b200_qmv_fusion))
        return fail(AFFON_B200_INVALID_ARG, "qmv_fused: null context or bad fusion descriptor");
    int rc = validate_desc(desc);
    if (rc) return rc;
    if (desc->numerical_policy == AFFON_B200_POLICY_EXACT_ONLY)
        return fail(AFFON_B200_POLICY_REJECTED,
                    "numericalPolicy exact_only rejects cuda_quantized_matmul (numerical class reassociated)");
    afb::QmvFusion f;
    f.x_mode = fusion->x_mode;
    f.epi = fusion->epilogue;
    f.h_out = fusion->h_out;
    f.ld_h_out = fusion->ld_h_out;
    f.ss_out = fusion->ss_out;
    f.act = static_cast<uint16_t *>(fusion->act);
    f.ld_act = fusion->ld_act;
    f.act_pair_order = fusion->act_pair_order;
    f.amax = fusion->amax;
    f.index_offset = fusion->index_offset;
    f.row_ss = fusion->row_ss;
    f.ss_tiles = fusion->ss_tiles;
    f.eps = fusion->eps;
    f.next_gamma = static_cast<const uint16_t *>(fusion->next_gamma);
    f.next_x = static_cast<uint16_t *>(fusion->next_x);
    f.ld_next_x = fusion->ld_next_x;
    f.next_pair_order = fusion->next_pair_order;
    if (f.row_ss && (f.ss_tiles <= 0 || f.ss_tiles * 16 != desc->x.cols || desc->x.rows > afb::kMaxQmvRows))
        return fail(AFFON_B200_INVALID_ARG, "qmv_fused: row scales need ss_tiles = K / 16");
    if (f.next_x && ((f.epi != 1 && f.epi != 4) || !f.next_gamma || f.ld_next_x < desc->w.rows))
        return fail(AFFON_B200_INVALID_ARG, "qmv_fused: next_x needs the residual epilogue, next_gamma and ld >= N");
    if (f.x_mode != 0 && f.x_mode != 1) return fail(AFFON_B200_INVALID_ARG, "qmv_fused: x_mode must be 0 or 1");
    if (f.epi < 0 || f.epi > 4) return fail(AFFON_B200_INVALID_ARG, "qmv_fused: unknown epilogue");
    if (((f.epi == 1 || f.epi == 4) && (!f.h_out || !f.ss_out)) || (f.epi == 2 && !f.act) || (f.epi == 3 && !f.amax) ||
        (f.epi == 0 && !y))
        return fail(AFFON_B200_INVALID_ARG, "qmv_fused: missing epilogue buffer");
    if (f.epi == 2 && desc->w.rows % 16) return fail(AFFON_B200_INVALID_SHAPE, "qmv_fused: silu*mul needs N % 16 == 0");
    if (!w || !s || !b || !x) return fail(AFFON_B200_INVALID_ARG, "qmv_fused: null buffer");
    char *fake = reinterpret_cast<char *>(uintptr_t(1) << 40);
    afb::QmmArgs a = make_args(desc, x, w, s, b, y ? y : fake);
    const char *why = "";
    if (!afb::qmv_supported(a, &why)) return fail(AFFON_B200_UNSUPPORTED, "qmv_fused: %s", why);
    // The fused tensor-parallel exchange (epilogue 4) runs on the stream-K plan.
    const afb::QmvPlan plan = afb::qmv_plan(a, ctx->num_sms, ctx->workspace_bytes, f.epi != 4);
    if (plan.splits < 1) return fail(AFFON_B200_UNSUPPORTED, "qmv_fused: no plan fits the context workspace");
    if (f.epi == 4) {
        const int64_t units = (a.N + plan.rows - 1) / plan.rows * plan.max_slots;
        const char *why = "";
        if (!afb::tp_bind_exchange(ctx, fusion->exchange_region, a.M, a.N, units, &f, &why))
            return fail(AFFON_B200_INVALID_ARG, "qmv_fused: %s", why);
    }
    DeviceGuard guard(ctx->device);
    cudaError_t e = afb::launch_qmv(a, plan, ctx->workspace, ctx->stream, &f, ctx->overlap);
    if (e != cudaSuccess) return cuda_fail(e, "qmv_fused launch");
    return AFFON_B200_OK;
}

int affon_b200_qmv_prep(affon_b200_ctx *ctx, int mode, const void *src, int64_t ld_src, const float *ss,
                        int ss_tiles, const void *gamma, float eps, int rows, int cols, int bits, void *dst,
                        int64_t ld_dst) {
    t_error.clear();
    if (!ctx || !src || !dst || rows <= 0 || rows > afb::kMaxQmvRows || cols <= 0 || cols % 8 || (bits != 4 && bits != 8) ||
        (mode != 0 && mode != 1) || ld_src % 8 || ld_dst % 8)
        return fail(AFFON_B200_INVALID_ARG, "qmv_prep: bad arguments");
    if (mode == 1 && (!ss || !gamma || ss_tiles <= 0))
        return fail(AFFON_B200_INVALID_ARG, "qmv_prep: rmsnorm needs ss and gamma");
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
    if (!al16(src) || !al16(dst) || (gamma && !al16(gamma))) return fail(AFFON_B200_INVALID_ARG, "qmv_prep: alignment");
    DeviceGuard guard(ctx->device);
    cudaError_t e = afb::launch_qmv_prep(src, ld_src, mode, ss, ss_tiles, static_cast<const uint16_t *>(gamma), eps,
                                         rows, cols, bits, static_cast<uint16_t *>(dst), ld_dst, ctx->stream,
                                         ctx->overlap);
    if (e != cudaSuccess) return cuda_fail(e, "qmv_prep launch");
    return AFFON_B200_OK;
}

int affon_b200_resid_norm(affon_b200_ctx *ctx, float *h, int64_t ld_h, const float *add, int64_t ld_add,
                          const void *gamma, float eps, int rows, int cols, int bits, void *dst, int64_t ld_dst) {
    t_error.clear();
    if (!ctx || !h || !gamma || !dst || rows <= 0 || rows > afb::kMaxQmvRows || cols <= 0 || cols % 8 ||
        cols > 8192 || (bits != 4 && bits != 8) || ld_h % 4 || (add && ld_add % 4) || ld_dst % 8)
        return fail(AFFON_B200_INVALID_ARG, "resid_norm: bad arguments (rows <= 32, cols % 8 == 0, cols <= 8192)");
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
    if (!al16(h) || (add && !al16(add)) || !al16(gamma) || !al16(dst))
        return fail(AFFON_B200_INVALID_ARG, "resid_norm: alignment");
    DeviceGuard guard(ctx->device);
    cudaError_t e = afb::launch_resid_norm(h, ld_h, add, ld_add, static_cast<const uint16_t *>(gamma), eps, rows, cols,
                                           bits, static_cast<uint16_t *>(dst), ld_dst, ctx->stream, ctx->overlap);
    if (e != cudaSuccess) return cuda_fail(e, "resid_norm launch");
    return AFFON_B200_OK;
}

int affon_b200_decode_attention(affon_b200_ctx *ctx, const affon_b200_attn_desc *d, const void *qkv, void *k_cache,
                                void *v_cache, const float *rope_cos, const float *rope_sin, const int *pos,
                                void *out) {
    t_error.clear();
    if (!ctx || !d || d->struct_size != sizeof(affon_b200_attn_desc))
        return fail(AFFON_B200_INVALID_ARG, "decode_attention: null context or bad descriptor");
    if (!qkv || !k_cache || !v_cache || !rope_cos || !rope_sin || !pos || !out)
        return fail(AFFON_B200_INVALID_ARG, "decode_attention: null buffer");
    if (d->head_dim != 128 || d->kv_heads <= 0 || d->q_heads % d->kv_heads ||
        (d->q_heads / d->kv_heads != 4 && d->q_heads / d->kv_heads != 8) || d->batch <= 0 || d->capacity <= 0)
        return fail(AFFON_B200_UNSUPPORTED, "decode_attention: head_dim 128 and 4 or 8 query heads per KV head");
    if ((reinterpret_cast<uintptr_t>(k_cache) % 16) || (reinterpret_cast<uintptr_t>(v_cache) % 16))
        return fail(AFFON_B200_INVALID_ARG, "decode_attention: caches must be 16-byte aligned");
    const size_t need = afb::attention_workspace_bytes(d->batch, d->kv_heads, d->q_heads, d->capacity, ctx->num_sms);
    if (need > ctx->workspace_bytes || size_t(d->batch) * d->kv_heads > size_t(afb::kMaxTiles / 2))
        return fail(AFFON_B200_UNSUPPORTED, "decode_attention: partials exceed the context workspace");
    afb::DecodeAttnArgs a{};
    a.qkv = qkv;
    a.ld_qkv = d->ld_qkv;
    a.q_off = d->q_offset;
    a.k_off = d->k_offset;
    a.v_off = d->v_offset;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.rope_cos = rope_cos;
    a.rope_sin = rope_sin;
    a.pos = pos;
    a.out = out;
    a.ld_out = d->ld_out;
    a.batch = d->batch;
    a.q_heads = d->q_heads;
    a.kv_heads = d->kv_heads;
    a.head_dim = d->head_dim;
    a.capacity = d->capacity;
    a.scale = d->scale;
    a.out_pair_order = d->out_pair_order;
    DeviceGuard guard(ctx->device);
    cudaError_t e = afb::launch_decode_attention(a, ctx->workspace, ctx->num_sms, ctx->stream, ctx->overlap);
    if (e != cudaSuccess) return cuda_fail(e, "decode_attention launch");
    return AFFON_B200_OK;
}

int affon_b200_embed(affon_b200_ctx *ctx, const void *table, int64_t ld_table, int64_t vocab, const int *tokens,
                     int batch, int dim, float *h, float *ss_out, unsigned long long *amax, const void *gamma,
                     void *x, int64_t ld_x, int pair_order) {
    t_error.clear();
    if (!ctx || !table || !tokens || !h || !ss_out || !amax || batch <= 0 || batch > afb::kMaxQmvRows || dim <= 0 ||
        dim % 16 || vocab <= 0 || (gamma && (!x || ld_x < dim)))
        return fail(AFFON_B200_INVALID_ARG, "embed: bad arguments (batch <= 32, dim % 16 == 0, vocab > 0)");
    DeviceGuard guard(ctx->device);
    cudaError_t e = afb::launch_embed(table, ld_table, vocab, tokens, batch, dim, h, ss_out, amax,
                                      static_cast<const uint16_t *>(gamma), static_cast<uint16_t *>(x), ld_x,
                                      pair_order, ctx->workspace, ctx->stream, ctx->overlap);
    if (e != cudaSuccess) return cuda_fail(e, "embed launch");
    return AFFON_B200_OK;
}

int affon_b200_argmax_finalize(affon_b200_ctx *ctx, const unsigned long long *amax, int batch, int *tokens,
                               int *history, int history_rows, int *pos, int *step) {
    t_error.clear();
    if (!ctx || !amax || !tokens || !pos || !step || batch <= 0 || batch > 1024 || (history && history_rows <= 0))
        return fail(AFFON_B200_INVALID_ARG, "argmax_finalize: bad arguments");
    DeviceGuard guard(ctx->device);
    cudaError_t e = afb::launch_finalize(amax, batch, tokens, history, history_rows, pos, step, ctx->stream,
                                         ctx->overlap);
    if (e != cudaSuccess) return cuda_fail(e, "finalize launch");
    return AFFON_B200_OK;
}

int affon_b200_compute_core_run_quantized_matmul_f32(const float *activation, size_t activation_count,
                                                     const uint32_t *weights, size_t weight_count, const float *scales,
                                                     size_t scale_count, const float *biases, size_t bias_count,
                                                     float *output, size_t output_count, size_t rows, size_t depth,
                                                     size_t columns, size_t bits, size_t group_size) {
    t_error.clear();
    // compute_core_cyna.zig:1013-1023 shape rules.
    if (rows == 0 || depth == 0 || columns == 0 || group_size == 0 || (bits != 2 && bits != 4 && bits != 8))
        return fail(AFFON_B200_INVALID_SHAPE, "InvalidShape");
    const size_t per_word = 32 / bits;
    if (depth % per_word || depth % group_size) return fail(AFFON_B200_INVALID_SHAPE, "InvalidShape");
    const size_t lim = size_t(1) << 40;
    if (rows > lim / depth || columns > lim / depth || rows > lim / columns)
        return fail(AFFON_B200_INVALID_SHAPE, "InvalidShape");
    if (activation_count != rows * depth || weight_count != columns * (depth / per_word) ||
        scale_count != columns * (depth / group_size) || bias_count != columns * (depth / group_size) ||
        output_count != rows * columns)
        return fail(AFFON_B200_INVALID_SHAPE, "InvalidShape");
    if (!activation || !weights || !scales || !biases || !output) return fail(AFFON_B200_INVALID_ARG, "null buffer");
    if (!t_default_ctx) {
        int rc = affon_b200_ctx_create(-1, nullptr, &t_default_ctx);
        if (rc) return rc;
    }
    affon_b200_qmm_desc d{};
    d.struct_size = sizeof d;
    d.bits = int32_t(bits);
    d.group_size = int64_t(group_size);
    d.x_dtype = d.param_dtype = d.y_dtype = AFFON_B200_F32;
    d.numerical_policy = AFFON_B200_POLICY_BACKEND_EQUIVALENT;
    const int64_t M = int64_t(rows), N = int64_t(columns), K = int64_t(depth);
    d.x = {M, K, K, 1, 0};
    d.w = {N, K / int64_t(per_word), K / int64_t(per_word), 1, 0};
    d.s = d.b = {N, K / int64_t(group_size), K / int64_t(group_size), 1, 0};
    d.y = {M, N, N, 1, 0};
    return affon_b200_qmm_host(t_default_ctx, &d, activation, weights, scales, biases, output);
}

}  // extern "C"
