// sm_100a primitives: mbarriers with bounded waits, TMA tensor loads, tcgen05
// (TMEM allocation, UMMA descriptors, MMA, commit, TMEM loads).  Written from
// the PTX ISA; no library code.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace afb {

// Error word written by device code; the host reads it through
// affon_b200_ctx_synchronize().  DEV_TIMEOUT: a bounded wait gave up;
// DEV_BOUNDS: a kernel read an index from device memory (a position, a token)
// that lies outside its buffer and skipped the access.
enum DeviceStatus : unsigned { DEV_OK = 0, DEV_TIMEOUT = 4, DEV_BOUNDS = 5 };

// Limits of the bounded waits: a pipeline-stage wait (mbarrier) and a wait on
// another CTA's or another GPU's arrival count.
constexpr uint64_t kStageWaitNs = 4000000000ull;
constexpr uint64_t kArrivalWaitNs = 4000000000ull;

AFB_DEVICE uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

AFB_DEVICE uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

AFB_DEVICE void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
AFB_DEVICE void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
AFB_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

AFB_DEVICE void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
AFB_DEVICE void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
AFB_DEVICE bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after
// `limit_ns` of wall time (checked every 256 polls), sets *abort and the
// device status word, and returns false.  Every other waiter sees *abort and
// leaves too, so no thread spins forever.
AFB_DEVICE bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned *status,
                          uint64_t limit_ns = kStageWaitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort) return false;
            if (globaltimer() - start > limit_ns) {
                *abort = 1;
                if (status) atomicExch(status, static_cast<unsigned>(DEV_TIMEOUT));
                return false;
            }
        }
    }
}

// Bounded wait that ignores the abort flag: used on the way out of a kernel
// to let copies already in flight land before shared memory is released.
// Returns false after `limit_ns`.
AFB_DEVICE bool mbar_wait_drain(uint64_t *bar, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer() - start > limit_ns) return false;
    }
}

// 2D tiled TMA load global -> shared, completion counted on `bar`.
AFB_DEVICE void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
// 3D tiled TMA load (coordinates innermost first).
AFB_DEVICE void tma_load_3d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
// The same load with an L2 cache policy (e.g. l2_evict_first()).
AFB_DEVICE void tma_load_2d_hint(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;"
        ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
        "l"(policy)
        : "memory");
}
// L2 policy for data read once per launch (streamed weights, caches): its
// lines are the first evicted, so streaming does not push out what the
// surrounding kernels reuse.
AFB_DEVICE uint64_t l2_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
AFB_DEVICE void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Programmatic dependent launch (the kernel was launched with the
// programmatic-stream-serialization attribute): pdl_wait() blocks until the
// preceding kernel in the stream has completed and its memory is visible;
// pdl_launch_dependents() lets the next kernel start launching once every CTA
// of this grid has issued it (or exited).  Both are no-ops without the
// attribute.
AFB_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
AFB_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Register reallocation between warpgroups (setmaxnreg): every warp of a
// warpgroup executes the same instruction.  An increase waits until other
// warpgroups have released enough registers, so the per-thread counts after
// all changes, times the threads of each warpgroup, must add up to no more
// than the block's launch allocation (threads x registers at launch).
template <int N>
AFB_DEVICE void regs_release() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N) : "memory");
}
template <int N>
AFB_DEVICE void regs_claim() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N) : "memory");
}

// Named barrier among `threads` threads (id 1..15; id 0 is __syncthreads).
AFB_DEVICE void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- tcgen05
AFB_DEVICE void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
AFB_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::); }
AFB_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
AFB_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
AFB_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 B, 8-row atoms of 1024 B): start address,
// leading byte offset (unused for this layout, 1), stride byte offset 1024 B
// between 8-row groups, version 1, layout SWIZZLE_128B (2).
AFB_DEVICE uint64_t umma_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;            // LBO (16-byte units)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;    // SBO
    d |= static_cast<uint64_t>(1u) << 46;            // version
    d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, f32 accumulate, both
// operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4)                                 // D format f32
           | (1u << 7)                               // A format bf16
           | (1u << 10)                              // B format bf16
           | (static_cast<uint32_t>(N >> 3) << 17)   // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);  // M / 16
}

AFB_DEVICE void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
AFB_DEVICE void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
AFB_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// 32 lanes x 32 bits, 32 consecutive columns per thread.
AFB_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
AFB_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same wait, with the 16 registers of a pending tmem_ld_32x32b_x16 as
// operands: every later use of them depends on the wait, so the compiler
// cannot move a use above it.
AFB_DEVICE void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

}  // namespace afb

// Host side: tensor-map encoding through the driver entry point (no -lcuda).
namespace afb {
bool encode_tensor_map_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner,
                          uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                          CUtensorMapSwizzle swizzle);
// Same, memoised per argument tuple (a bounded process-wide cache), so
// repeated launches on the same buffers skip the driver call.  The returned
// map stays valid until the process exits.
const CUtensorMap *cached_tensor_map_2d(CUtensorMapDataType dtype, const void *base, uint64_t inner, uint64_t outer,
                                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                                        CUtensorMapSwizzle swizzle);
// A memoised 3D map: dims innermost first, byte strides of dims 1 and 2 (any
// order; each a multiple of 16), box innermost first.
const CUtensorMap *cached_tensor_map_3d(CUtensorMapDataType dtype, const void *base, uint64_t d0, uint64_t d1,
                                        uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0,
                                        uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle);
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device, size).
cudaError_t ensure_smem_attr(const void *kernel, int bytes);

// cudaLaunchKernelEx with the optional cooperative (every CTA resident at
// once) and programmatic-dependent-launch attributes.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool coop,
                      bool pdl, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (coop) {
        attr[n].id = cudaLaunchAttributeCooperative;
        attr[n].val.cooperative = 1;
        ++n;
    }
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}
}  // namespace afb
