// Tensor-parallel group of a context: one NCCL communicator per rank (one
// process per GPU), made non-blocking so every wait on it is bounded on the
// host: initialisation, each collective's enqueue, stream completion and
// teardown poll ncclCommGetAsyncError against a deadline and abort the
// communicator when it passes, returning AFFON_B200_TIMEOUT instead of
// hanging on a peer that died or never joined.
//
// The unique id that rank 0 creates is sealed (magic, NCCL id, FNV-1a hash)
// so that a corrupted or truncated id is rejected before NCCL would try to
// connect to whatever address it decodes to.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or the file named by
// AFFON_NCCL_LIBRARY): a process that already loaded NCCL (PyTorch does)
// shares that copy, and the library itself does not depend on NCCL unless a
// tensor-parallel entry point is called.
#include <dlfcn.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include <nccl.h>

#include "../../include/affon_b200.h"
#include "internal.h"
#include "sm100.cuh"

namespace afb {

namespace {

struct NcclApi {
    bool loaded = false;
    std::string error;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*GetVersion)(int *) = nullptr;
};

NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = nullptr;
        const char *env = getenv("AFFON_NCCL_LIBRARY");
        if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);  // the process's copy
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char *e = dlerror();
            api.error = std::string("cannot load NCCL (libnccl.so.2): ") + (e ? e : "unknown error");
            return;
        }
        bool ok = true;
        auto sym = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) {
                ok = false;
                api.error = std::string("NCCL lacks ") + name;
            }
        };
        sym(api.GetUniqueId, "ncclGetUniqueId");
        sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(api.CommAbort, "ncclCommAbort");
        sym(api.CommFinalize, "ncclCommFinalize");
        sym(api.CommDestroy, "ncclCommDestroy");
        sym(api.AllReduce, "ncclAllReduce");
        sym(api.AllGather, "ncclAllGather");
        sym(api.GetErrorString, "ncclGetErrorString");
        sym(api.GetVersion, "ncclGetVersion");
        api.loaded = ok;
    });
    return api;
}

// Sealed unique id: [0,4) magic, [4,8) format version, [8,136) ncclUniqueId,
// [136,144) FNV-1a 64-bit hash of bytes [0,136).
constexpr uint32_t kIdMagic = 0x50544641u;  // "AFTP"
constexpr uint32_t kIdVersion = 1;
static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
static_assert(AFFON_B200_TP_ID_BYTES == 144, "sealed id size");

uint64_t fnv1a(const unsigned char *p, size_t n) {
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

bool id_ok(const void *id) {
    const unsigned char *p = static_cast<const unsigned char *>(id);
    uint32_t magic, version;
    uint64_t hash;
    memcpy(&magic, p, 4);
    memcpy(&version, p + 4, 4);
    memcpy(&hash, p + 136, 8);
    return magic == kIdMagic && version == kIdVersion && hash == fnv1a(p, 136);
}

int fmt_error(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fmt_error(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return set_error(status, buf);
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct TpState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    double timeout_s = 60.0;
    bool aborted = false;
    // Exchange buffers of the fused row-parallel reduction: this rank's
    // buffer and every rank's mapping of theirs (CUDA IPC), each holding two
    // regions of [world][max_rows][max_cols] f32 plus arrival flags.
    void *xbuf = nullptr;
    void *peer[kTpMaxWorld] = {};
    size_t region_bytes = 0, recv_bytes = 0;
    int max_rows = 0;
    int64_t max_cols = 0;
};

namespace {

// Abort the communicator (peers see their collectives fail) and mark the
// group unusable.
void abort_comm(TpState *t) {
    if (t->comm && !t->aborted) nccl().CommAbort(t->comm);
    t->comm = nullptr;
    t->aborted = true;
}

// Poll the communicator until its pending operation has left the
// ncclInProgress state, or the deadline passes (then abort).
int wait_comm(TpState *t, double timeout_s, const char *what) {
    const auto t0 = Clock::now();
    for (;;) {
        ncclResult_t st = ncclInProgress;
        ncclResult_t r = nccl().CommGetAsyncError(t->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return AFFON_B200_OK;
        if (st != ncclInProgress) {
            abort_comm(t);
            return fmt_error(AFFON_B200_CUDA_ERROR, "tensor parallel %s: NCCL error %d (%s); group aborted", what,
                             int(st), nccl().GetErrorString(st));
        }
        if (std::chrono::duration<double>(Clock::now() - t0).count() > timeout_s) {
            abort_comm(t);
            return fmt_error(AFFON_B200_TIMEOUT, "tensor parallel %s: no progress within %.1f s; group aborted", what,
                             timeout_s);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int need_group(affon_b200_ctx *ctx) {
    if (!ctx) return set_error(AFFON_B200_INVALID_ARG, "null context");
    if (!ctx->tp) return set_error(AFFON_B200_INVALID_ARG, "the context has no tensor-parallel group (tp_init)");
    if (ctx->tp->aborted) return set_error(AFFON_B200_CUDA_ERROR, "the tensor-parallel group was aborted");
    return AFFON_B200_OK;
}

struct DevScope {
    int prev = -1;
    explicit DevScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DevScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

void tp_release(affon_b200_ctx *ctx) {
    if (!ctx || !ctx->tp) return;
    TpState *t = ctx->tp;
    // Every rank stops touching the exchange buffers before it leaves: the
    // caller synchronises (tp_synchronize) before tearing the group down.
    for (int r = 0; r < t->world; ++r)
        if (t->peer[r] && r != t->rank) cudaIpcCloseMemHandle(t->peer[r]);
    if (t->xbuf) cudaFree(t->xbuf);
    if (t->comm && !t->aborted) {
        // Finalize flushes outstanding work; bounded like every other wait
        // (wait_comm aborts the communicator when it fails).
        ncclResult_t r = nccl().CommFinalize(t->comm);
        if (r != ncclSuccess && r != ncclInProgress)
            abort_comm(t);
        else if (wait_comm(t, t->timeout_s, "finalize") == AFFON_B200_OK)
            nccl().CommDestroy(t->comm);
    }
    delete t;
    ctx->tp = nullptr;
}

bool tp_bind_exchange(affon_b200_ctx *ctx, int region, int64_t rows, int64_t cols, int64_t units, QmvFusion *f,
                      const char **why) {
    TpState *t = ctx ? ctx->tp : nullptr;
    if (!t || t->aborted) { *why = "no live tensor-parallel group"; return false; }
    if (!t->xbuf) { *why = "no exchange buffers (affon_b200_tp_exchange_reserve)"; return false; }
    if (region < 0 || region > 1) { *why = "exchange region must be 0 or 1"; return false; }
    if (rows > t->max_rows || cols > t->max_cols) { *why = "projection larger than the reserved exchange"; return false; }
    if (units > kTpMaxUnits) { *why = "too many row units for the exchange flags"; return false; }
    f->tp_world = t->world;
    f->tp_rank = t->rank;
    for (int r = 0; r < t->world; ++r) {
        char *base = static_cast<char *>(t->peer[r]) + region * t->region_bytes;
        f->tp_recv[r] = reinterpret_cast<float *>(base);
        f->tp_flags_peer[r] = reinterpret_cast<unsigned *>(base + t->recv_bytes);
    }
    f->tp_flags_local = f->tp_flags_peer[t->rank];
    return true;
}

}  // namespace afb

using afb::nccl;

extern "C" {

int affon_b200_tp_id_check(const void *id) {
    afb::clear_error();
    if (!id) return afb::set_error(AFFON_B200_INVALID_ARG, "tp: null unique id");
    if (!afb::id_ok(id))
        return afb::set_error(AFFON_B200_INVALID_ARG, "tp: unique id is corrupted (magic, version or checksum)");
    return AFFON_B200_OK;
}

int affon_b200_tp_unique_id(void *out) {
    afb::clear_error();
    if (!out) return afb::set_error(AFFON_B200_INVALID_ARG, "tp: null output");
    if (!nccl().loaded) return afb::set_error(AFFON_B200_UNSUPPORTED, nccl().error.c_str());
    ncclUniqueId uid;
    ncclResult_t r = nccl().GetUniqueId(&uid);
    if (r != ncclSuccess)
        return afb::fmt_error(AFFON_B200_CUDA_ERROR, "ncclGetUniqueId: %s", nccl().GetErrorString(r));
    unsigned char *p = static_cast<unsigned char *>(out);
    memcpy(p, &afb::kIdMagic, 4);
    memcpy(p + 4, &afb::kIdVersion, 4);
    memcpy(p + 8, &uid, 128);
    const uint64_t h = afb::fnv1a(p, 136);
    memcpy(p + 136, &h, 8);
    return AFFON_B200_OK;
}

int affon_b200_tp_init(affon_b200_ctx *ctx, int rank, int world, const void *unique_id, double timeout_s) {
    afb::clear_error();
    if (!ctx) return afb::set_error(AFFON_B200_INVALID_ARG, "null context");
    if (ctx->tp) return afb::set_error(AFFON_B200_INVALID_ARG, "tp_init: the context already has a group");
    if (world < 1 || rank < 0 || rank >= world)
        return afb::fmt_error(AFFON_B200_INVALID_ARG, "tp_init: rank %d outside a group of %d", rank, world);
    if (!(timeout_s > 0)) return afb::set_error(AFFON_B200_INVALID_ARG, "tp_init: timeout must be positive");
    int rc = affon_b200_tp_id_check(unique_id);
    if (rc) return rc;
    if (!nccl().loaded) return afb::set_error(AFFON_B200_UNSUPPORTED, nccl().error.c_str());
    afb::DevScope dev(ctx->device);
    auto *t = new afb::TpState;
    t->rank = rank;
    t->world = world;
    t->timeout_s = timeout_s;
    ncclUniqueId uid;
    memcpy(&uid, static_cast<const unsigned char *>(unique_id) + 8, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every wait is polled against a deadline
    ncclResult_t r = nccl().CommInitRankConfig(&t->comm, world, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (t->comm) nccl().CommAbort(t->comm);
        delete t;
        return afb::fmt_error(AFFON_B200_CUDA_ERROR, "ncclCommInitRankConfig: %s", nccl().GetErrorString(r));
    }
    rc = afb::wait_comm(t, timeout_s, "init");
    if (rc) {
        std::string msg = affon_b200_last_error();
        delete t;
        return afb::set_error(rc, msg.c_str());
    }
    ctx->tp = t;
    return AFFON_B200_OK;
}

int affon_b200_tp_exchange_reserve(affon_b200_ctx *ctx, int max_rows, int64_t max_cols) {
    afb::clear_error();
    int rc = afb::need_group(ctx);
    if (rc) return rc;
    if (max_rows <= 0 || max_rows > afb::kMaxQmvRows || max_cols <= 0)
        return afb::set_error(AFFON_B200_INVALID_ARG, "tp_exchange_reserve: 0 < rows <= 32, cols > 0");
    afb::TpState *t = ctx->tp;
    if (t->world > afb::kTpMaxWorld) return afb::set_error(AFFON_B200_UNSUPPORTED, "tp_exchange_reserve: world > 8");
    if (t->xbuf) return afb::set_error(AFFON_B200_INVALID_ARG, "tp_exchange_reserve: already reserved");
    afb::DevScope dev(ctx->device);
    const size_t recv = (size_t(t->world) * max_rows * size_t(max_cols) * 4 + 255) / 256 * 256;
    const size_t region = recv + size_t(afb::kTpMaxUnits) * 4;
    cudaError_t e = cudaMalloc(&t->xbuf, 2 * region);
    if (e != cudaSuccess) return afb::set_cuda_error(e, "tp exchange cudaMalloc");
    if ((e = cudaMemset(t->xbuf, 0, 2 * region)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess)
        return afb::set_cuda_error(e, "tp exchange clear");
    // Share the buffer: every rank's IPC handle, gathered through NCCL.
    cudaIpcMemHandle_t mine;
    if ((e = cudaIpcGetMemHandle(&mine, t->xbuf)) != cudaSuccess) return afb::set_cuda_error(e, "cudaIpcGetMemHandle");
    char *dsend = nullptr, *drecv = nullptr;
    if ((e = cudaMalloc(&dsend, sizeof mine)) != cudaSuccess ||
        (e = cudaMalloc(&drecv, sizeof mine * t->world)) != cudaSuccess)
        return afb::set_cuda_error(e, "tp exchange handles");
    cudaIpcMemHandle_t all[afb::kTpMaxWorld];
    e = cudaMemcpy(dsend, &mine, sizeof mine, cudaMemcpyHostToDevice);
    ncclResult_t r = e == cudaSuccess ? nccl().AllGather(dsend, drecv, sizeof mine, ncclUint8, t->comm, ctx->stream)
                                      : ncclInvalidArgument;
    if (r != ncclSuccess && r != ncclInProgress) {
        cudaFree(dsend);
        cudaFree(drecv);
        return afb::fmt_error(AFFON_B200_CUDA_ERROR, "tp exchange all-gather: %s", nccl().GetErrorString(r));
    }
    rc = afb::wait_comm(t, t->timeout_s, "exchange all-gather");
    if (rc == AFFON_B200_OK) {
        rc = affon_b200_tp_synchronize(ctx, t->timeout_s);
        if (rc == AFFON_B200_OK && (e = cudaMemcpy(all, drecv, sizeof mine * t->world, cudaMemcpyDeviceToHost)) != cudaSuccess)
            rc = afb::set_cuda_error(e, "tp exchange handles read");
    }
    cudaFree(dsend);
    cudaFree(drecv);
    if (rc) return rc;
    for (int p = 0; p < t->world; ++p) {
        if (p == t->rank) {
            t->peer[p] = t->xbuf;
            continue;
        }
        if ((e = cudaIpcOpenMemHandle(&t->peer[p], all[p], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
            return afb::set_cuda_error(e, "cudaIpcOpenMemHandle");
    }
    t->region_bytes = region;
    t->recv_bytes = recv;
    t->max_rows = max_rows;
    t->max_cols = max_cols;
    return AFFON_B200_OK;
}

int affon_b200_tp_rank(const affon_b200_ctx *ctx) { return ctx && ctx->tp ? ctx->tp->rank : -1; }
int affon_b200_tp_world(const affon_b200_ctx *ctx) { return ctx && ctx->tp ? ctx->tp->world : 0; }

int affon_b200_tp_allreduce(affon_b200_ctx *ctx, void *buf, size_t count, int dtype, int op) {
    afb::clear_error();
    int rc = afb::need_group(ctx);
    if (rc) return rc;
    if (!buf && count) return afb::set_error(AFFON_B200_INVALID_ARG, "tp_allreduce: null buffer");
    ncclDataType_t dt;
    switch (dtype) {
    case AFFON_B200_F32: dt = ncclFloat32; break;
    case AFFON_B200_BF16: dt = ncclBfloat16; break;
    case AFFON_B200_U64: dt = ncclUint64; break;
    default: return afb::set_error(AFFON_B200_INVALID_DTYPE, "tp_allreduce: dtype must be f32, bf16 or u64");
    }
    if (op != AFFON_B200_REDUCE_SUM && op != AFFON_B200_REDUCE_MAX)
        return afb::set_error(AFFON_B200_INVALID_ARG, "tp_allreduce: op must be sum or max");
    if (dtype == AFFON_B200_U64 && op != AFFON_B200_REDUCE_MAX)
        return afb::set_error(AFFON_B200_INVALID_ARG, "tp_allreduce: u64 supports max only");
    afb::DevScope dev(ctx->device);
    afb::TpState *t = ctx->tp;
    ncclResult_t r = nccl().AllReduce(buf, buf, count, dt, op == AFFON_B200_REDUCE_SUM ? ncclSum : ncclMax, t->comm,
                                      ctx->stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        afb::abort_comm(t);
        return afb::fmt_error(AFFON_B200_CUDA_ERROR, "ncclAllReduce: %s; group aborted", nccl().GetErrorString(r));
    }
    return afb::wait_comm(t, t->timeout_s, "all-reduce enqueue");
}

int affon_b200_tp_allreduce_bf16(affon_b200_ctx *ctx, void *buf, size_t count) {
    return affon_b200_tp_allreduce(ctx, buf, count, AFFON_B200_BF16, AFFON_B200_REDUCE_SUM);
}

int affon_b200_tp_synchronize(affon_b200_ctx *ctx, double timeout_s) {
    afb::clear_error();
    int rc = afb::need_group(ctx);
    if (rc) return rc;
    afb::DevScope dev(ctx->device);
    afb::TpState *t = ctx->tp;
    const double limit = timeout_s > 0 ? timeout_s : t->timeout_s;
    const auto t0 = afb::Clock::now();
    for (;;) {
        cudaError_t q = cudaStreamQuery(ctx->stream);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return afb::set_cuda_error(q, "tp_synchronize");
        ncclResult_t st = ncclSuccess;
        if (nccl().CommGetAsyncError(t->comm, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
            afb::abort_comm(t);
            return afb::fmt_error(AFFON_B200_CUDA_ERROR, "tp_synchronize: NCCL error %d (%s); group aborted", int(st),
                                  nccl().GetErrorString(st));
        }
        if (std::chrono::duration<double>(afb::Clock::now() - t0).count() > limit) {
            afb::abort_comm(t);
            return afb::fmt_error(AFFON_B200_TIMEOUT, "tp_synchronize: stream not done within %.1f s; group aborted",
                                  limit);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return affon_b200_ctx_synchronize(ctx);
}

int affon_b200_tp_abort(affon_b200_ctx *ctx) {
    afb::clear_error();
    if (!ctx || !ctx->tp) return AFFON_B200_OK;
    afb::DevScope dev(ctx->device);
    afb::abort_comm(ctx->tp);
    return AFFON_B200_OK;
}

int affon_b200_tp_destroy(affon_b200_ctx *ctx) {
    afb::clear_error();
    if (!ctx || !ctx->tp) return AFFON_B200_OK;
    afb::DevScope dev(ctx->device);
    afb::tp_release(ctx);
    return AFFON_B200_OK;
}

}  // extern "C"
