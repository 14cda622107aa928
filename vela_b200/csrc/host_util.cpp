#include "host_util.h"
#include <cudaTypedefs.h>
#include <mutex>
#include <string>
#include <vector>

namespace vela {
namespace {
PFN_cuTensorMapEncodeTiled_v12000 encodeFn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) throw Error(VELA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver)");
    return fn;
}
CUtensorMapSwizzle swz(Swz s) {
    switch (s) {
        case Swz::B32: return CU_TENSOR_MAP_SWIZZLE_32B;
        case Swz::B64: return CU_TENSOR_MAP_SWIZZLE_64B;
        case Swz::B128: return CU_TENSOR_MAP_SWIZZLE_128B;
        default: return CU_TENSOR_MAP_SWIZZLE_NONE;
    }
}
std::mutex g_mu;
std::vector<const void*> g_symbols;
}  // namespace

CUtensorMap tmap2d(const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer, uint64_t ld_bytes,
                   uint32_t boxInner, uint32_t boxOuter, Swz s) {
    CUtensorMap m;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld_bytes};
    cuuint32_t box[2] = {boxInner, boxOuter};
    cuuint32_t es[2] = {1, 1};
    CUresult r = encodeFn()(&m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz(s),
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        throw Error(VELA_ERR_ARG, "cuTensorMapEncodeTiled(2d) failed: code " + std::to_string(int(r)) + " dims " + std::to_string(inner) + "x" +
                                  std::to_string(outer) + " ld " + std::to_string(ld_bytes));
    return m;
}
CUtensorMap tmap_nhwc(const void* base, uint64_t B, uint64_t H, uint64_t W, uint64_t C,
                      uint32_t boxC, uint32_t boxW, uint32_t boxH, uint32_t boxB, uint32_t stride, Swz s) {
    CUtensorMap m;
    cuuint64_t dims[4] = {C, W, H, B};
    cuuint64_t strides[3] = {C * 4, W * C * 4, H * W * C * 4};
    cuuint32_t box[4] = {boxC, boxW, boxH, boxB};
    cuuint32_t es[4] = {1, stride, stride, 1};
    CUresult r = encodeFn()(&m, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz(s),
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(VELA_ERR_ARG, "cuTensorMapEncodeTiled(nhwc) failed: code " + std::to_string(int(r)));
    return m;
}

int current_device() { int d = 0; VELA_CUDA(cudaGetDevice(&d)); return d; }
int sm_count() {
    static std::atomic<int> cache[64];
    const int d = current_device();
    if (d < 64) { const int c = cache[d].load(std::memory_order_relaxed); if (c) return c; }
    int n = 0; VELA_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d));
    if (d < 64) cache[d].store(n, std::memory_order_relaxed);
    return n;
}

int blocks_per_sm(const void* kernel, int threads, size_t smem) {
    struct Entry { int dev; const void* k; int threads; size_t smem; int blocks; };
    static std::mutex mu;
    static std::vector<Entry> cache;
    const int d = current_device();
    {
        std::lock_guard<std::mutex> lk(mu);
        for (const Entry& e : cache) if (e.dev == d && e.k == kernel && e.threads == threads && e.smem == smem) return e.blocks;
    }
    int n = 0;
    VELA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem));
    n = n > 0 ? n : 1;
    std::lock_guard<std::mutex> lk(mu);
    cache.push_back(Entry{d, kernel, threads, smem, n});
    return n;
}

void register_error_word(const void* symbol) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto* s : g_symbols) if (s == symbol) return;
    g_symbols.push_back(symbol);
}
unsigned* device_error_word(const void* symbol) {
    register_error_word(symbol);
    void* p = nullptr;
    VELA_CUDA(cudaGetSymbolAddress(&p, symbol));
    return static_cast<unsigned*>(p);
}
unsigned read_device_errors(bool clear) {
    std::vector<const void*> syms;
    { std::lock_guard<std::mutex> lk(g_mu); syms = g_symbols; }
    unsigned all = 0;
    for (auto* s : syms) {
        unsigned v = 0;
        VELA_CUDA(cudaMemcpyFromSymbol(&v, s, sizeof(v)));
        all |= v;
        if (clear && v) { unsigned z = 0; VELA_CUDA(cudaMemcpyToSymbol(s, &z, sizeof(z))); }
    }
    return all;
}
}  // namespace vela
