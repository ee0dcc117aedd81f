// Host helpers for sm_100a kernels: tensor-map encoding via the driver entry
// point (the library does not link libcuda directly).
#include <cudaTypedefs.h>

#include <deque>
#include <map>
#include <mutex>
#include <tuple>

#include "sm100.cuh"

namespace afb {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool encode_tensor_map_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner,
                          uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                          CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

namespace {
using MapKey = std::tuple<int, uintptr_t, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t, int>;
struct MapCache {
    std::mutex mu;
    std::map<MapKey, CUtensorMap *> maps;
    std::deque<MapKey> order;
    std::deque<CUtensorMap *> retired;  // evicted maps are kept alive (a launch may still hold a copy)
};
MapCache &map_cache() {
    static MapCache *c = new MapCache;
    return *c;
}
}  // namespace

const CUtensorMap *cached_tensor_map_2d(CUtensorMapDataType dtype, const void *base, uint64_t inner, uint64_t outer,
                                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                                        CUtensorMapSwizzle swizzle) {
    MapKey key{int(dtype), reinterpret_cast<uintptr_t>(base), inner, outer, row_stride_bytes, box_inner, box_outer,
               int(swizzle)};
    MapCache &c = map_cache();
    std::lock_guard<std::mutex> lock(c.mu);
    auto it = c.maps.find(key);
    if (it != c.maps.end()) return it->second;
    CUtensorMap *m = new CUtensorMap;
    if (!encode_tensor_map_2d(m, dtype, base, inner, outer, row_stride_bytes, box_inner, box_outer, swizzle)) {
        delete m;
        return nullptr;
    }
    if (c.order.size() >= 4096) {
        MapKey old = c.order.front();
        c.order.pop_front();
        auto o = c.maps.find(old);
        if (o != c.maps.end()) {
            c.retired.push_back(o->second);
            if (c.retired.size() > 4096) {
                delete c.retired.front();
                c.retired.pop_front();
            }
            c.maps.erase(o);
        }
    }
    c.maps.emplace(key, m);
    c.order.push_back(key);
    return m;
}

namespace {
using Map3Key = std::tuple<int, uintptr_t, uint64_t, uint64_t, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t,
                           uint32_t, int>;
struct Map3Cache {
    std::mutex mu;
    std::map<Map3Key, CUtensorMap *> maps;
    std::deque<Map3Key> order;
    std::deque<CUtensorMap *> retired;  // evicted maps are kept alive (a launch may still hold a copy)
};
Map3Cache &map3_cache() {
    static Map3Cache *c = new Map3Cache;
    return *c;
}
}  // namespace

const CUtensorMap *cached_tensor_map_3d(CUtensorMapDataType dtype, const void *base, uint64_t d0, uint64_t d1,
                                        uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0,
                                        uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle) {
    Map3Key key{int(dtype), reinterpret_cast<uintptr_t>(base), d0, d1, d2, stride1_bytes, stride2_bytes, b0, b1, b2,
                int(swizzle)};
    Map3Cache &c = map3_cache();
    std::lock_guard<std::mutex> lock(c.mu);
    auto it = c.maps.find(key);
    if (it != c.maps.end()) return it->second;
    auto fn = encode_fn();
    if (!fn) return nullptr;
    CUtensorMap *m = new CUtensorMap;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, dtype, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        delete m;
        return nullptr;
    }
    if (c.order.size() >= 4096) {
        Map3Key old = c.order.front();
        c.order.pop_front();
        auto o = c.maps.find(old);
        if (o != c.maps.end()) {
            c.retired.push_back(o->second);
            if (c.retired.size() > 4096) {
                delete c.retired.front();
                c.retired.pop_front();
            }
            c.maps.erase(o);
        }
    }
    c.maps.emplace(key, m);
    c.order.push_back(key);
    return m;
}

cudaError_t ensure_smem_attr(const void *kernel, int bytes) {
    static std::mutex mu;
    static std::map<std::tuple<const void *, int>, int> done;  // (kernel, device) -> configured bytes
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_tuple(kernel, dev);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done[key] = bytes;
    return e;
}

}  // namespace afb
