// Host helpers shared by the kernel translation units: TMA tensor maps,
// per-device error words, small integer utilities.
#pragma once
#include "status.h"
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <cstddef>

namespace vela {

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

enum class Swz { None = 0, B32 = 1, B64 = 2, B128 = 3 };
// Tiled tensor map over a row-major 2-D array: `inner` elements per row (contiguous), `outer` rows,
// `ld_bytes` between rows; box of boxInner x boxOuter elements.  Out-of-range boxes read zeros.
CUtensorMap tmap2d(const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer, uint64_t ld_bytes,
                   uint32_t boxInner, uint32_t boxOuter, Swz swz);
// 4-D map over an NHWC int32 image [B][H][W][C] with element strides (1, s, s, 1) along (C, W, H, B).
CUtensorMap tmap_nhwc(const void* base, uint64_t B, uint64_t H, uint64_t W, uint64_t C,
                      uint32_t boxC, uint32_t boxW, uint32_t boxH, uint32_t boxB, uint32_t stride, Swz swz);

// Address (on the current device) of a translation unit's __device__ error word; cached per device.
unsigned* device_error_word(const void* symbol);
// Read and optionally clear every registered error word on the current device (OR of all).
unsigned read_device_errors(bool clear);
void register_error_word(const void* symbol);

int current_device();
int sm_count();
// Blocks of `kernel` resident on one SM at `threads` threads and `smem` dynamic shared bytes (at least 1), on the
// current device; cached.  Grids of this many blocks per SM run in one wave.
int blocks_per_sm(const void* kernel, int threads, size_t smem);

// Per-launch options of the kernels with bounded waits (GEMM, attention).
struct LaunchOpts {
    unsigned* err = nullptr;       // device error word the kernel reports a timeout into; null: the kernel file's own word
    long long wait_limit = 0;      // SM clock cycles before a wait gives up; 0: the default (WAIT_LIMIT_CYCLES)
    int stall = 0;                 // failure-path tests only: the TMA producers issue nothing, so every wait runs out
};

// Runs `f` (an idempotent per-device setup such as cudaFuncSetAttribute) until it has succeeded once on the current
// device; `done` is a zero-initialised static array of 64 flags owned by the caller.  Threads may race into `f`
// together, which is harmless for idempotent setups; the flags themselves are atomic.
template <class F> void once_per_device(std::atomic<int>* done, F&& f) {
    const int d = current_device();
    if (d < 64 && done[d].load(std::memory_order_acquire)) return;
    f();
    if (d < 64) done[d].store(1, std::memory_order_release);
}
}  // namespace vela
